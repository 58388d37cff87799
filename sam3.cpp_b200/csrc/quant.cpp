// Host quantisers for the ggml block formats used by .ggml model files
// (examples/quantize.cpp:195-265 calls ggml_quantize_chunk for these types).
// The rounding steps are ggml's reference quantisers (ggml-quants.c,
// quantize_row_q4_0_ref / q4_1_ref / q8_0_ref), restated here:
//   q4_0: d = v / -8 with v the element of largest |x|; q = min(15, trunc(x/d + 8.5))
//   q4_1: d = (max - min) / 15; m = min; q = min(15, trunc((x - m)/d + 0.5))
//   q8_0: d = amax / 127; q = roundf(x / d)
// with 1/d computed once per block (0 when d == 0) and d, m stored as f16.
#include <math.h>
#include <string.h>

#include <cuda_fp16.h>

#include "kernels.h"

namespace s3b {

static uint16_t f2h(float f) {
  const __half h = __float2half_rn(f);
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

void quantize_row_host(int type, const float* x, int64_t n, uint8_t* dst) {
  const int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; ++b) {
    const float* v = x + b * 32;
    if (type == QT_Q4_0) {
      float amax = 0.f, vmax = 0.f;
      for (int j = 0; j < 32; ++j)
        if (fabsf(v[j]) > amax) {
          amax = fabsf(v[j]);
          vmax = v[j];
        }
      const float d = vmax / -8.0f;
      const float id = d != 0.f ? 1.0f / d : 0.0f;
      uint8_t* o = dst + b * 18;
      const uint16_t dh = f2h(d);
      memcpy(o, &dh, 2);
      for (int j = 0; j < 16; ++j) {
        const float x0 = v[j] * id, x1 = v[16 + j] * id;
        int q0 = (int)(int8_t)(x0 + 8.5f), q1 = (int)(int8_t)(x1 + 8.5f);
        q0 = q0 < 15 ? q0 : 15;
        q1 = q1 < 15 ? q1 : 15;
        o[2 + j] = (uint8_t)(q0 | (q1 << 4));
      }
    } else if (type == QT_Q4_1) {
      float vmin = v[0], vmax = v[0];
      for (int j = 1; j < 32; ++j) {
        if (v[j] < vmin) vmin = v[j];
        if (v[j] > vmax) vmax = v[j];
      }
      const float d = (vmax - vmin) / 15.0f;
      const float id = d != 0.f ? 1.0f / d : 0.0f;
      uint8_t* o = dst + b * 20;
      const uint16_t dh = f2h(d), mh = f2h(vmin);
      memcpy(o, &dh, 2);
      memcpy(o + 2, &mh, 2);
      for (int j = 0; j < 16; ++j) {
        const float x0 = (v[j] - vmin) * id, x1 = (v[16 + j] - vmin) * id;
        int q0 = (int)(int8_t)(x0 + 0.5f), q1 = (int)(int8_t)(x1 + 0.5f);
        q0 = q0 < 15 ? q0 : 15;
        q1 = q1 < 15 ? q1 : 15;
        o[4 + j] = (uint8_t)(q0 | (q1 << 4));
      }
    } else {  // Q8_0
      float amax = 0.f;
      for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
      const float d = amax / 127.0f;
      const float id = d != 0.f ? 1.0f / d : 0.0f;
      uint8_t* o = dst + b * 34;
      const uint16_t dh = f2h(d);
      memcpy(o, &dh, 2);
      for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(int8_t)roundf(v[j] * id);
    }
  }
}

}  // namespace s3b
