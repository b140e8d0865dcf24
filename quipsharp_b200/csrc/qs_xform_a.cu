// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(0, false)
QS_DEFINE_XFFT_RUNNERS(0, true)
QS_DEFINE_XFWHT_RUNNERS(false)
QS_DEFINE_XFWHT_RUNNERS(true)
}  // namespace qs
