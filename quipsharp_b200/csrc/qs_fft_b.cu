// Explicit instantiations of the FFT kernels (split for parallel compilation).
#include "qs_fft.cuh"

namespace qs {
QS_DEFINE_FFT_RUNNERS(true, 13)
QS_DEFINE_FFT_RUNNERS(true, 17)
QS_DEFINE_FFT_RUNNERS(true, 19)
}  // namespace qs
