// Explicit instantiations of the transform kernels (split for parallel compilation).
#include "qs_xform.cuh"

namespace qs {
QS_DEFINE_XFFT_RUNNERS(23, false)
QS_DEFINE_XFFT_RUNNERS(23, true)
QS_DEFINE_XFFT_RUNNERS(29, false)
QS_DEFINE_XFFT_RUNNERS(29, true)
}  // namespace qs
