// rcu_gemm.cu -- prefill GEMM entry (n_tok > 8). Placeholder until the tcgen05 kernel
// lands: reports RCU_ERR_UNSUPPORTED so the dispatcher runs the GEMV in 8-token slices.
#include "rcu_kernels.h"

namespace rcu {
int launch_gemm(rcu_ctx *ctx, const ActsView &, const HostJob *, int) {
    return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: not available");
}
}  // namespace rcu
