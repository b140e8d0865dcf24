// Explicit instantiations of the FFT kernels (split for parallel compilation).
#include "qs_fft.cuh"

namespace qs {
QS_DEFINE_FFT_RUNNERS(false, 0)
QS_DEFINE_FFT_RUNNERS(true, 0)
QS_DEFINE_FFT_RUNNERS(true, 11)
}  // namespace qs
