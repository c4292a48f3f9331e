// Dequantization of the relaid Q4_K / Q8_0 weight tiles into f16 pairs, shared by the tcgen05 GEMM and the GEMV:
// packed f16 arithmetic (lop3 / prmt into the mantissa of 1024, then one fma), every weight rounded once to f16.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace gck {

GCK_DEV uint32_t hsub2_u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b), *reinterpret_cast<__half2 *>(&c));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t hmul2_u(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

constexpr uint32_t kMagic = 0x64006400u;   // f16 pair (1024, 1024): OR-ing an integer below 1024 into a half adds it
constexpr uint32_t kP64 = 0x64646464u;     // byte source of prmt: 0x64 in every byte
constexpr uint32_t kH1024 = 0x64006400u;
constexpr uint32_t kH1152 = 0x64806480u;   // 1024 + 128
constexpr uint32_t kH16th = 0x2C002C00u;   // 1/16
constexpr uint32_t kHm64 = 0xD400D400u;    // -64

// One Q4_K quant word of the relaid tile: 8 nibbles of k = 0..7 at bit positions 0, 16, 4, 20, 8, 24, 12, 28, so
// that masking gives f16 pairs of consecutive k: (1024 + q) for the nibbles at bits 0/16 and 8/24, (1024 + 16q) for
// those at 4/20 and 12/28 -> exact q by one subtraction or one fma, then q * S + O with one rounding.
GCK_DEV void q4_word(uint32_t w, uint32_t S, uint32_t O, uint32_t *o) {
  const uint32_t w8 = w >> 8;
  const uint32_t a = (w & 0x000F000Fu) | kMagic, b = (w & 0x00F000F0u) | kMagic;
  const uint32_t c = (w8 & 0x000F000Fu) | kMagic, d = (w8 & 0x00F000F0u) | kMagic;
  o[0] = hfma2_u(hsub2_u(a, kH1024), S, O);
  o[1] = hfma2_u(hfma2_u(b, kH16th, kHm64), S, O);
  o[2] = hfma2_u(hsub2_u(c, kH1024), S, O);
  o[3] = hfma2_u(hfma2_u(d, kH16th, kHm64), S, O);
}
// One Q8_0 quant word of the relaid tile: 4 bytes q + 128 of k = 0..3 -> two f16 pairs (q0, q1) * D, (q2, q3) * D
GCK_DEV void q8_word(uint32_t w, uint32_t D, uint32_t *o) {
  o[0] = hmul2_u(hsub2_u(prmt(w, kP64, 0x5140u), kH1152), D);
  o[1] = hmul2_u(hsub2_u(prmt(w, kP64, 0x5342u), kH1152), D);
}

// Q4_K super-block header words (bytes 4..15 of the block: 12 packed six-bit scales and mins) -> the scales and mins
// of sub-blocks g0 and g0 + 1 (g0 even) as exact f16 pairs, then S = d * sc and O = -dmin * m, one rounding each (the
// products are exact in f32, so this equals rounding the f32 product). dd = (d, d), mm = (-dmin, -dmin).
// Sub-blocks 0-3: low 6 bits of bytes 0-3 (scales) / 4-7 (mins); 4-7: low / high nibbles of bytes 8-11 with the top
// 2 bits of bytes 0-3 / 4-7.
GCK_DEV void q4k_pair_scales(const uint4 &hdr, int g0, uint32_t dd, uint32_t mm, uint32_t &S01, uint32_t &O01) {
  uint32_t scw, mw;
  if (g0 < 4) {
    scw = hdr.y & 0x3F3F3F3Fu;
    mw = hdr.z & 0x3F3F3F3Fu;
  } else {
    scw = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    mw = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  }
  // bytes g0 % 4 and g0 % 4 + 1 into the low bytes of two halves whose high bytes are 0x64: (1024 + x, 1024 + y)
  const uint32_t sel = (g0 & 2) ? 0x5342u : 0x5140u;
  S01 = hmul2_u(hsub2_u(prmt(scw, kP64, sel), kH1024), dd);
  O01 = hmul2_u(hsub2_u(prmt(mw, kP64, sel), kH1024), mm);
}

}  // namespace gck
