// GGUF weight formats of pkg/quant/dequant.go, decoded four elements at a
// time.  Shared by the device dequantization (quant.cu) and, compiled as
// plain C++, by the test that checks this exact code on the host against the
// oracle, so the arithmetic and indexing the kernel runs are verified bit for
// bit without a GPU.
//
// Type codes and block geometry are GGUF's (pkg/gguf/format.go:40-58,
// :117-149).  Every value is computed in float32 with one rounding per
// operation and no fused multiply-add, like the reference compiled for amd64:
//   F32   (0)  raw float32                                   dequant.go:369-373
//   F16   (1)  fp16ToFp32                                   :9-41, :50-56
//   Q4_0  (2)  18 B / 32: d, 16 B nibbles (low = element 2i); d*(q-8)      :99-119
//   Q4_1  (3)  20 B / 32: d, min, 16 B nibbles; d*q + min                 :141-163
//   Q5_0  (6)  22 B / 32: d, 32 high bits (bit k = element k), nibbles;
//              d*(q-16)                                                     :167-199
//   Q5_1  (7)  24 B / 32: d, min, high bits, nibbles; d*q + min           :203-233
//   Q8_0  (8)  34 B / 32: d, 32 int8; d*q                                 :68-85
//   Q4_K (12)  144 B / 256: d, dmin, 12 B of 6-bit scales and mins, 128 B
//              nibbles (sub-block j = elements 32j..32j+31, low nibble first);
//              (d*sc[j])*q - dmin*m[j]                                      :237-300
//   Q6_K (14)  210 B / 256: 128 B low nibbles, 64 B 2-bit highs, 16 int8
//              scales, d; (d*scale[k/16])*(q-32)                           :304-344
// These layouts are the reference's and differ from ggml's for Q5_0/Q5_1 and
// the K-quants; the reference's are followed.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define QF_HD __host__ __device__ __forceinline__
#else
#define QF_HD inline
#endif

namespace glc {
namespace qf {

enum : int { F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q4_K = 12, Q6_K = 14 };

// Elements per block and bytes per block; 0 for an unknown type.
QF_HD int block_elems(int type) {
  switch (type) {
    case F32: case F16: return 1;
    case Q4_0: case Q4_1: case Q5_0: case Q5_1: case Q8_0: return 32;
    case Q4_K: case Q6_K: return 256;
    default: return 0;
  }
}
QF_HD int block_bytes(int type) {
  switch (type) {
    case F32: return 4;
    case F16: return 2;
    case Q4_0: return 18;
    case Q4_1: return 20;
    case Q5_0: return 22;
    case Q5_1: return 24;
    case Q8_0: return 34;
    case Q4_K: return 144;
    case Q6_K: return 210;
    default: return 0;
  }
}

// float32 arithmetic with one rounding each (never contracted into an FMA).
#if defined(__CUDA_ARCH__)
QF_HD float mul(float a, float b) { return __fmul_rn(a, b); }
QF_HD float add(float a, float b) { return __fadd_rn(a, b); }
QF_HD float sub(float a, float b) { return __fsub_rn(a, b); }
QF_HD float bits_to_float(uint32_t u) { return __uint_as_float(u); }
QF_HD int clz32(uint32_t x) { return __clz(x); }
#else
// The host build compiles with -ffp-contract=off: each operator is one IEEE
// float32 operation.
inline float mul(float a, float b) { return a * b; }
inline float add(float a, float b) { return a + b; }
inline float sub(float a, float b) { return a - b; }
inline float bits_to_float(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline int clz32(uint32_t x) { return x ? __builtin_clz(x) : 32; }
#endif

// fp16ToFp32 (dequant.go:9-41) in integer operations: a subnormal half is
// normalised as the reference's shift loop does; NaN payloads are kept.
QF_HD float half_to_float(uint32_t h) {
  const uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu, bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign << 31;
    } else {
      const int s = clz32(m) - 21;  // shifts until bit 10 is set
      m = (m << s) & 0x3ffu;
      bits = (sign << 31) | (static_cast<uint32_t>(1 - s + 127 - 15) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = (sign << 31) | 0x7f800000u | (m << 13);
  } else {
    bits = (sign << 31) | ((e + 127 - 15) << 23) | (m << 13);
  }
  return bits_to_float(bits);
}

// Little-endian 16-bit field; every format keeps these at even offsets of
// even-sized blocks, so a 2-byte aligned source suffices.
QF_HD uint32_t u16(const uint8_t* p) {
#if defined(__CUDA_ARCH__)
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p));
#else
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
#endif
}

QF_HD uint32_t nibble(const uint8_t* q, int k) {  // element k of nibble-packed codes, low nibble first
  const uint32_t b = q[k >> 1];
  return (k & 1) ? (b >> 4) : (b & 0x0fu);
}

// Q4_K's 6-bit scale and min of sub-block j (dequant.go:260-283).
QF_HD void q4k_scale_min(const uint8_t* s, int j, uint32_t* sc, uint32_t* m) {
  if (j < 4) {
    *sc = s[j] & 63u;
    *m = s[j + 4] & 63u;
  } else {
    const int t = j - 4;
    const uint32_t lo_s = s[8 + (t >> 1)], lo_m = s[10 + (t >> 1)];
    *sc = ((t & 1) ? (lo_s >> 4) : (lo_s & 0x0fu)) | ((static_cast<uint32_t>(s[t]) >> 6) << 4);
    *m = ((t & 1) ? (lo_m >> 4) : (lo_m & 0x0fu)) | ((static_cast<uint32_t>(s[4 + t]) >> 6) << 4);
  }
}

// Elements 4g .. 4g+3 of a tensor of `type` stored at `src` (4g in bounds;
// for block types the tensor holds whole blocks).
QF_HD void dequant4(const uint8_t* src, int type, size_t g, float v[4]) {
  if (type == F32) {
    const uint8_t* p = src + 16 * g;
    for (int i = 0; i < 4; ++i) v[i] = bits_to_float(u16(p + 4 * i) | (u16(p + 4 * i + 2) << 16));
    return;
  }
  if (type == F16) {
    const uint8_t* p = src + 8 * g;
    for (int i = 0; i < 4; ++i) v[i] = half_to_float(u16(p + 2 * i));
    return;
  }
  const int be = block_elems(type);
  const size_t groups = static_cast<size_t>(be / 4);
  const size_t blk = g / groups;
  const int k0 = static_cast<int>(g % groups) * 4;  // first element inside the block
  const uint8_t* b = src + blk * static_cast<size_t>(block_bytes(type));
  switch (type) {
    case Q8_0: {
      const float d = half_to_float(u16(b));
      const uint32_t q = u16(b + 2 + k0) | (u16(b + 4 + k0) << 16);
      for (int i = 0; i < 4; ++i) v[i] = mul(d, static_cast<float>(static_cast<int8_t>((q >> (8 * i)) & 0xffu)));
      return;
    }
    case Q4_0: {
      const float d = half_to_float(u16(b));
      for (int i = 0; i < 4; ++i) v[i] = mul(d, static_cast<float>(static_cast<int>(nibble(b + 2, k0 + i)) - 8));
      return;
    }
    case Q4_1: {
      const float d = half_to_float(u16(b)), mn = half_to_float(u16(b + 2));
      for (int i = 0; i < 4; ++i) v[i] = add(mul(d, static_cast<float>(nibble(b + 4, k0 + i))), mn);
      return;
    }
    case Q5_0: {
      const float d = half_to_float(u16(b));
      const uint32_t qh = u16(b + 2) | (u16(b + 4) << 16);
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i;
        const uint32_t q = nibble(b + 6, k) | (((qh >> k) & 1u) << 4);
        v[i] = mul(d, static_cast<float>(static_cast<int>(q) - 16));
      }
      return;
    }
    case Q5_1: {
      const float d = half_to_float(u16(b)), mn = half_to_float(u16(b + 2));
      const uint32_t qh = u16(b + 4) | (u16(b + 6) << 16);
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i;
        const uint32_t q = nibble(b + 8, k) | (((qh >> k) & 1u) << 4);
        v[i] = add(mul(d, static_cast<float>(q)), mn);
      }
      return;
    }
    case Q4_K: {
      const float d = half_to_float(u16(b)), dmin = half_to_float(u16(b + 2));
      const int j = k0 >> 5;  // the four elements share one sub-block
      uint32_t sc, m;
      q4k_scale_min(b + 4, j, &sc, &m);
      const float scale = mul(d, static_cast<float>(sc)), mnv = mul(dmin, static_cast<float>(m));
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i;
        // sub-block j holds its 32 elements in bytes 16j .. 16j+15
        const uint32_t q = nibble(b + 16 + 16 * j, k & 31);
        v[i] = sub(mul(scale, static_cast<float>(q)), mnv);
      }
      return;
    }
    case Q6_K: {
      const float d = half_to_float(u16(b + 208));
      // the four elements share one qh byte and one scale (k0 % 4 == 0)
      const float scale = mul(d, static_cast<float>(static_cast<int8_t>(b[192 + (k0 >> 4)])));
      const uint32_t hb = b[128 + (k0 >> 2)];
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i;
        const uint32_t q = nibble(b, k) | (((hb >> (2 * i)) & 3u) << 4);
        v[i] = mul(scale, static_cast<float>(static_cast<int>(q) - 32));
      }
      return;
    }
    default:
      for (int i = 0; i < 4; ++i) v[i] = 0.f;
  }
}

}  // namespace qf
}  // namespace glc
