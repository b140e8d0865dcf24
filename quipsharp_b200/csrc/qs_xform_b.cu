// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(11, false)
QS_DEFINE_XFFT_RUNNERS(11, true)
QS_DEFINE_XFFT_RUNNERS(13, false)
QS_DEFINE_XFFT_RUNNERS(13, true)
}  // namespace qs
