"""GRPO example: python examples/run_grpo.py --config configs/grpo_tiny_cpu.yaml [k=v ...]"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from lumenrl_b200.trainer.main import main  # noqa: E402

if __name__ == "__main__":
    main()
