// Explicit instantiations of the FFT kernels (split for parallel compilation).
#include "qs_fft.cuh"

namespace qs {
QS_DEFINE_FFT_RUNNERS(true, 43)
}  // namespace qs
