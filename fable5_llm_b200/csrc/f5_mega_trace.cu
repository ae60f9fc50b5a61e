// The traced instance of the persistent decode-step kernel: f5_mega.cu
// compiled again with its per-op globaltimer marks in (k_mega_traced,
// launched by f5_ctx_trace_step only).  The step kernel itself carries no
// mark: the kernel is one function whose speed follows its code size.
#define F5_MEGA_TRACE 1
#include "f5_mega.cu"
