// qtb_quant.cpp -- host-side weight encoders of the engine (plain C++, no
// device code).  Each one produces the exact bytes of the format the decode
// kernels consume:
//   qtb_quantize_int8     per-row absmax int8 + f32 scale, the reference's
//                         qwen_quantize_bf16_to_int8 (qwen_tts_kernels.c:2143-2238;
//                         its x86 vector path rounds to nearest-even)
//   qtb_quantize_q4_0     the reference's weighted-LSQ q4_0 encoder
//                         (qwen_quantize_bf16_to_q4_0, qwen_tts_kernels.c:2662-2726)
//   qtb_quantize_int4g32  asymmetric int4, group 32, fp16 scale + fp16 zero
//                         (the engine's own format; the reference has none)
#include "../../include/qwen3tts_b200.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

void par_rows(int n, const std::function<void(int, int)> &fn) {
  unsigned hw = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  int nt = std::min<int>((int)hw, std::max(1, n / 64));
  if (nt <= 1) { fn(0, n); return; }
  std::vector<std::thread> th;
  for (int i = 0; i < nt; i++)
    th.emplace_back(fn, (int)((long long)n * i / nt), (int)((long long)n * (i + 1) / nt));
  for (auto &t : th) t.join();
}

inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// f32 -> IEEE binary16 with the rounding rule of the reference's portable
// converter (qwen_tts_kernels.h qwen_f32_to_f16): round half up on the
// discarded bits, subnormals rounded to nearest, overflow to inf.
uint16_t f32_to_f16_ref(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int32_t e = (int32_t)((bits >> 23) & 0xff) - 127 + 15;
  uint32_t m = bits & 0x7fffffu;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000u;
    const uint32_t shift = (uint32_t)(14 - e);
    uint16_t sub = (uint16_t)(m >> shift);
    if ((m >> (shift - 1)) & 1u) sub++;
    return (uint16_t)(sign | sub);
  }
  uint16_t out = (uint16_t)(sign | ((uint32_t)e << 10) | (m >> 13));
  if (m & 0x1000u) out++;
  return out;
}

// IEEE binary16 round-to-nearest-even (the int4g32 format's scale / zero).
uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000u) {  // below the smallest normal half: round to subnormal units of 2^-24
    if (ax <= 0x33000000u) return (uint16_t)sign;  // <= 2^-25 -> 0 (ties to even)
    const int e = (int)(ax >> 23);
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const int sh = 126 - e;  // 14..24
    uint32_t res = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), halfway = 1u << (sh - 1);
    if (rem > halfway || (rem == halfway && (res & 1u))) res++;
    return (uint16_t)(sign | res);
  }
  uint32_t res = ((ax >> 13) - (112u << 10));
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (res & 1u))) res++;
  return (uint16_t)(sign | res);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t em = h & 0x7fffu;
  uint32_t bits;
  if (em >= 0x7c00u) bits = sign | 0x7f800000u | ((em & 0x3ffu) << 13);
  else if (em >= 0x400u) bits = sign | ((em + ((127u - 15u) << 10)) << 13);
  else if (em == 0) bits = sign;
  else {
    int shift = 0;
    uint32_t m = em;
    while (!(m & 0x400u)) { m <<= 1; shift++; }
    bits = sign | ((uint32_t)(127 - 15 - shift) << 23) | ((m & 0x3ffu) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

extern "C" int qtb_quantize_int8(const uint16_t *src, int rows, int cols, int8_t *dst, float *scale) {
  if (!src || !dst || !scale || rows <= 0 || cols <= 0) return QTB_E_INVALID;
  par_rows(rows, [&](int r0, int r1) {
    for (int r = r0; r < r1; r++) {
      const uint16_t *row = src + (size_t)r * cols;
      float amax = 0.f;
      for (int k = 0; k < cols; k++) amax = std::max(amax, std::fabs(bf16_to_f32(row[k])));
      // the reference is built with -ffast-math, which turns amax / 127.0f into
      // amax * (1/127.0f): reproduce that rounding for identical scales
      const float s = amax * (1.0f / 127.0f);
      scale[r] = s;
      const float inv = (s > 0) ? 127.0f / amax : 0.0f;
      for (int k = 0; k < cols; k++) {
        int v = (int)std::nearbyint(bf16_to_f32(row[k]) * inv);
        dst[(size_t)r * cols + k] = (int8_t)std::min(127, std::max(-128, v));
      }
    }
  });
  return 0;
}

extern "C" int qtb_quantize_q4_0(const uint16_t *src, int rows, int cols, uint8_t *dst_blocks) {
  if (!src || !dst_blocks || rows <= 0 || cols <= 0 || cols % 32) return QTB_E_INVALID;
  const int nb = cols / 32;
  par_rows(rows, [&](int r0, int r1) {
    for (int r = r0; r < r1; r++)
      for (int b = 0; b < nb; b++) {
        const uint16_t *blk = src + (size_t)r * cols + b * 32;
        float v[32];
        float amax = 0.f, vmax = 0.f;
        for (int i = 0; i < 32; i++) {
          v[i] = bf16_to_f32(blk[i]);
          const float a = std::fabs(v[i]);
          if (a > amax) { amax = a; vmax = v[i]; }
        }
        const float isc = (vmax != 0.0f) ? -8.0f / vmax : 0.0f;
        int q[32];
        double num = 0.0, den = 0.0;
        for (int i = 0; i < 32; i++) {
          int t = (int)std::round(v[i] * isc);
          t = std::min(7, std::max(-8, t));
          q[i] = t;
          const double w = (double)v[i] * v[i];
          num += w * v[i] * t;
          den += w * (double)t * t;
        }
        const float s = (den > 0.0) ? (float)(num / den) : 0.0f;
        uint8_t *out = dst_blocks + ((size_t)r * nb + b) * 18;
        const uint16_t h = f32_to_f16_ref(s);
        out[0] = (uint8_t)(h & 0xff);
        out[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 16; i++) out[2 + i] = (uint8_t)((q[2 * i] + 8) | ((q[2 * i + 1] + 8) << 4));
      }
  });
  return 0;
}

extern "C" int qtb_quantize_int4g32(const uint16_t *src, int rows, int cols, uint8_t *codes, uint16_t *scale,
                                    uint16_t *zero) {
  if (!src || !codes || !scale || !zero || rows <= 0 || cols <= 0 || cols % 32) return QTB_E_INVALID;
  const int ng = cols / 32;
  par_rows(rows, [&](int r0, int r1) {
    for (int r = r0; r < r1; r++)
      for (int g = 0; g < ng; g++) {
        float v[32];
        float mn = INFINITY, mx = -INFINITY;
        for (int i = 0; i < 32; i++) {
          v[i] = bf16_to_f32(src[(size_t)r * cols + g * 32 + i]);
          mn = std::min(mn, v[i]);
          mx = std::max(mx, v[i]);
        }
        float sc = (mx - mn) / 15.0f;
        float z;
        if (!(sc > 0.0f)) { sc = 1.0f; z = -mn; }
        else z = -mn / sc;
        const uint16_t hs = f32_to_f16_rne(sc), hz = f32_to_f16_rne(z);
        const float s16 = f16_to_f32(hs), z16 = f16_to_f32(hz);
        scale[(size_t)r * ng + g] = hs;
        zero[(size_t)r * ng + g] = hz;
        for (int i = 0; i < 32; i += 2) {
          int q0 = (int)std::nearbyint(v[i] / s16 + z16), q1 = (int)std::nearbyint(v[i + 1] / s16 + z16);
          q0 = std::min(15, std::max(0, q0));
          q1 = std::min(15, std::max(0, q1));
          codes[(size_t)r * (cols / 2) + g * 16 + i / 2] = (uint8_t)(q0 | (q1 << 4));
        }
      }
  });
  return 0;
}

extern "C" uint16_t qtb_f32_to_f16_rne(float f) { return f32_to_f16_rne(f); }
