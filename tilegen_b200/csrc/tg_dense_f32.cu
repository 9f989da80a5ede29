// Explicit instantiation of the SpMM / SDDMM host dispatch for float (see tg_dense_host.cuh).
#include "tg_dense_host.cuh"

namespace tg {

template size_t dense_ws_bytes<float>(int64_t, int64_t, int64_t, const tg_sched&, bool);
template int dense_run<float>(bool, const tg_csr&, const float*, const float*, float*, int64_t, const tg_sched&, void*,
                              size_t, cudaStream_t);

}  // namespace tg
