// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(41, false)
QS_DEFINE_XFFT_RUNNERS(41, true)
QS_DEFINE_XFFT_RUNNERS(43, false)
QS_DEFINE_XFFT_RUNNERS(43, true)
}  // namespace qs
