// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(17, false)
QS_DEFINE_XFFT_RUNNERS(17, true)
QS_DEFINE_XFFT_RUNNERS(19, false)
QS_DEFINE_XFFT_RUNNERS(19, true)
}  // namespace qs
