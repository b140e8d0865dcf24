// Explicit instantiations of the FFT kernels (split for parallel compilation).
#include "qs_fft.cuh"

namespace qs {
QS_DEFINE_FFT_RUNNERS(true, 31)
QS_DEFINE_FFT_RUNNERS(true, 37)
}  // namespace qs
