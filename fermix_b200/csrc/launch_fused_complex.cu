// Register-panel and generic one-block-per-matrix kernels for complex64 / complex128.
#include "launch_fused.inl"

namespace fxh {
#define FXH_INST(T)                                                               \
  template int plan_fused<T, false>(int64_t, int, int, Plan&);                    \
  template int plan_fused<T, true>(int64_t, int, int, Plan&);                     \
  template int launch_fused<T, false>(cudaStream_t, Job<T>, void*, size_t);       \
  template int launch_fused<T, true>(cudaStream_t, Job<T>, void*, size_t);
FXH_FOR_COMPLEX(FXH_INST)
}  // namespace fxh
