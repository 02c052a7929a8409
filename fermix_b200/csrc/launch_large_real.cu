// Blocked LU / Parlett-Reid engines (n > 256) for float32 / float64.
#include "launch_large.inl"

namespace fxh {
#define FXH_INST(T)                                                                 \
  template size_t lg_ws_bytes<T>(int64_t, int);                                     \
  template int run_large_lu<T>(cudaStream_t, Job<T>, void*, size_t, bool, bool);    \
  template int run_large_pf<T>(cudaStream_t, Job<T>, void*, size_t);
FXH_FOR_REAL(FXH_INST)
}  // namespace fxh
