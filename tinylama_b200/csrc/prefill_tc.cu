// prefill_tc.cu -- causal GQA prefill attention on the tcgen05 tensor cores (bf16 in, fp32
// accumulate in TMEM).  Placeholder until the kernel lands: reports "not covered" so the
// caller uses the fp32 CUDA-core kernel.
#include "internal.h"

namespace tl {
cudaError_t launch_prefill_tc(const PrefillArgs &a, cudaStream_t s) {
    (void)a;
    (void)s;
    return cudaErrorNotSupported;
}
}  // namespace tl
