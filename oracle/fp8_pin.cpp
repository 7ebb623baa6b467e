// Known-answer source for the oracle's e4m3 rounding: CUDA's own host-side
// float -> e4m3 conversion (cuda_fp8.h, saturating, round-to-nearest-even),
// wrapped for ctypes. Test infrastructure only.
#include <cuda_fp8.h>

#include <cstdint>

extern "C" void pin_f32_to_e4m3_array(const float* in, uint8_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = static_cast<uint8_t>(
        __nv_cvt_float_to_fp8(in[i], __NV_SATFINITE, __NV_E4M3));
}
