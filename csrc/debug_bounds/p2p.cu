// The p2p.cu NVLink kernels compiled into lumenrl_b200._C_bounds (built with
// -DLRL_DEBUG_BOUNDS: every peer and signal-area access bounds-checked).
#include "../comm/p2p.cu"
