// Explicit instantiation of the SpMM / SDDMM host dispatch for double (see tg_dense_host.cuh).
#include "tg_dense_host.cuh"

namespace tg {

template size_t dense_ws_bytes<double>(int64_t, int64_t, int64_t, const tg_sched&, bool);
template int dense_run<double>(bool, const tg_csr&, const double*, const double*, double*, int64_t, const tg_sched&, void*,
                              size_t, cudaStream_t);

}  // namespace tg
