// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(31, false)
QS_DEFINE_XFFT_RUNNERS(31, true)
QS_DEFINE_XFFT_RUNNERS(37, false)
QS_DEFINE_XFFT_RUNNERS(37, true)
}  // namespace qs
