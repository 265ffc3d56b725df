// lumenrl_b200._C_bounds: the NVLink communication kernels built with
// -DLRL_DEBUG_BOUNDS.  Every peer and signal-area access is checked against
// the extent of the buffer it goes through; a violation is skipped and its
// site code recorded in the per-device bounds status word (bounds_status()).
// Selected instead of the ordinary comm ops with LRL_DEBUG_BOUNDS=1.
#include <torch/extension.h>

#include "comm/comm_api.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { lrl::def_comm_ops(m); }
