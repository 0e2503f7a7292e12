// Device helpers shared by the attention kernels (dense "flat" tiles and
// block-sparse tiles).
#pragma once

#include "icsa_kernels.cuh"
#include "icsa_tcgen05.cuh"

namespace icsa {
namespace attn {

constexpr int kChunkBytes = 128 * 128;     // one 64-wide K chunk of a 128-row operand (SW128)
constexpr float kRescaleThreshold = 8.0f;  // lazy O rescale: p may reach 2^8

// Error codes written to *err (first writer wins).
enum : int {
  kErrQ = 0x101, kErrKFull = 0x102, kErrVFull = 0x103, kErrKEmpty = 0x104, kErrVEmpty = 0x105,
  kErrSFull = 0x106, kErrSEmpty = 0x107, kErrPFull = 0x108, kErrPvDone = 0x109, kErrDrain = 0x10A
};

// Warp-uniform bounded wait: every lane polls the barrier (so each lane
// acquires the phase), and the decision to give up is taken by the whole warp
// so that warp-collective tcgen05 instructions stay converged.
ICSA_DEV bool warp_mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag) {
  bool done = mbar_try_wait(bar, parity);
  uint64_t t0 = 0;
  uint32_t it = 0;
  while (!__all_sync(0xffffffffu, done)) {
    if (!done) done = mbar_try_wait(bar, parity);
    bool give_up = *abort_flag != 0;
    if ((threadIdx.x & 31) == 0 && (++it & 63u) == 0u) {
      const uint64_t now = global_timer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > 1000000000ull) {
        report_error(err, code);
        *abort_flag = 1;
        give_up = true;
      }
    }
    if (__any_sync(0xffffffffu, give_up)) return false;
  }
  return true;
}

// Bounded wait used when draining at exit: ignores the abort flag so that
// copies still in flight land before the CTA's shared memory is released.
ICSA_DEV void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 1000000000ull) {
      report_error(err, kErrDrain);
      return;
    }
  }
}

// 2^x on the multi-function unit (flushes subnormal results to zero, which
// only affects probabilities below 2^-126 of the row maximum).
ICSA_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input maximum (sm_100 max.f32 with three sources).
ICSA_DEV float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Max over 128 registers: 8 independent chains of three-input maxima (a single
// chain would serialise the instructions).
ICSA_DEV float max128(const float (&s)[128]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(s[i], s[i + 8]);
#pragma unroll
  for (int c = 16; c < 128; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3(m[i], s[c + i], s[c + 8 + i]);
  return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}
ICSA_DEV void tmem_load_row128(uint32_t taddr, float (&s)[128]) {
  uint32_t r[4][32];
#pragma unroll
  for (int c = 0; c < 4; ++c) tc::tmem_ld32(taddr + c * 32, r[c]);
  tc::tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[c][e]);
}

ICSA_DEV float load_alpha(const AttnParams& p, int b, int token, int h, int d) {
  const long long off = b * p.alpha_strides[0] + token * p.alpha_strides[1] + h * p.alpha_strides[2] +
                        d * p.alpha_strides[3];
  if (p.alpha_dtype == ICSA_F32) return reinterpret_cast<const float*>(p.alpha)[off];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.alpha)[off]);
}


// Residual for 32 consecutive features [d0, d0+32) of one output row:
// x = bf16(o) + out_c * alpha, with the reference's dtype rounding (attention
// outputs are bf16; out_compress and out_compress*alpha are bf16 when the
// reference computes them in bf16).  oc_row == nullptr: plain attention,
// x = bf16(o).
ICSA_DEV void residual32(const AttnParams& p, int b, int token, int h, const float* oc_row, int d0,
                         const float (&o)[32], float (&x)[32]) {
  if (oc_row == nullptr) {
#pragma unroll
    for (int e = 0; e < 32; ++e) x[e] = bf16_round(o[e]);
    return;
  }
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int d = d0 + e;
    float cval = oc_row[d];
    if (p.outc_bf16) cval = bf16_round(cval);
    const float a = (p.alpha_mode == ICSA_ALPHA_SCALAR) ? p.alpha_scalar : load_alpha(p, b, token, h, d);
    float ca = cval * a;
    if (p.ca_bf16) ca = bf16_round(ca);
    x[e] = bf16_round(o[e]) + ca;
  }
}

// out_c * alpha for a scalar alpha, with the same rounding as residual32; it
// is the same for every row of a query block, so kernels compute it once per
// block (row of D values) and then use residual32_ca.
ICSA_DEV float ca_scalar(const AttnParams& p, float cval) {
  if (p.outc_bf16) cval = bf16_round(cval);
  float ca = cval * p.alpha_scalar;
  if (p.ca_bf16) ca = bf16_round(ca);
  return ca;
}
ICSA_DEV void residual32_ca(const float* ca_row, int d0, const float (&o)[32], float (&x)[32]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) x[e] = bf16_round(o[e]) + ca_row[d0 + e];
}

// The same, stored to the output row as the output dtype.
ICSA_DEV void store_out32(const AttnParams& p, int b, int token, int h, const float* oc_row, int d0,
                          const float (&o)[32], size_t out_row) {
  float x[32];
  residual32(p, b, token, h, oc_row, d0, o, x);
  if (p.out_dtype == ICSA_BF16) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + out_row + d0;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 u;
      u.x = pack_bf16x2(x[v * 8 + 0], x[v * 8 + 1]);
      u.y = pack_bf16x2(x[v * 8 + 2], x[v * 8 + 3]);
      u.z = pack_bf16x2(x[v * 8 + 4], x[v * 8 + 5]);
      u.w = pack_bf16x2(x[v * 8 + 6], x[v * 8 + 7]);
      reinterpret_cast<uint4*>(dst)[v] = u;
    }
  } else {
    float* dst = reinterpret_cast<float*>(p.out) + out_row + d0;
#pragma unroll
    for (int v = 0; v < 8; ++v)
      reinterpret_cast<float4*>(dst)[v] = make_float4(x[v * 4], x[v * 4 + 1], x[v * 4 + 2], x[v * 4 + 3]);
  }
}

// Packed two-lane fp32 arithmetic (sm_100 f32x2 instructions).
ICSA_DEV void ffma2(float& x, float& y, float a0, float a1, float b0, float b1, float c0, float c1) {
  asm("{.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;}"
      : "=f"(x), "=f"(y)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
ICSA_DEV void fadd2(float& x, float& y, float a0, float a1, float b0, float b1) {
  asm("{.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;}"
      : "=f"(x), "=f"(y)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
ICSA_DEV void fmul2(float& x, float& y, float a0, float a1, float b0, float b1) {
  asm("{.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;}"
      : "=f"(x), "=f"(y)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x for two values on the FMA/ALU pipes, to take load off the
// multi-function unit.  Range reduction x = n + f with n = rint(x) obtained
// by the 1.5 * 2^23 rounding shift, f in [-0.5, 0.5]; 2^f by a cubic whose
// coefficients were fitted (iteratively reweighted least squares on the
// relative error over [-0.5, 0.5]) for this kernel, max relative error
// 7.6e-5, far below the 2^-9 of the bf16 probabilities it feeds; then n is
// added to the exponent field.  Inputs below -126 are clamped, so a masked
// -inf gives ~1e-38 instead of 0, which vanishes against any unmasked term.
constexpr float kExp2C0 = 0.99992835521698f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.24260826408863068f;
constexpr float kExp2C3 = 0.05517039820551872f;
constexpr float kRoundShift = 12582912.0f;  // 1.5 * 2^23

ICSA_DEV void exp2_poly2(float& a, float& b) {
  a = fmaxf(a, -126.0f);
  b = fmaxf(b, -126.0f);
  float ta, tb, ja, jb, fa, fb, pa, pb;
  fadd2(ta, tb, a, b, kRoundShift, kRoundShift);
  fadd2(ja, jb, ta, tb, -kRoundShift, -kRoundShift);
  ffma2(fa, fb, ja, jb, -1.0f, -1.0f, a, b);
  ffma2(pa, pb, kExp2C3, kExp2C3, fa, fb, kExp2C2, kExp2C2);
  ffma2(pa, pb, pa, pb, fa, fb, kExp2C1, kExp2C1);
  ffma2(pa, pb, pa, pb, fa, fb, kExp2C0, kExp2C0);
  a = __int_as_float(__float_as_int(pa) + ((__float_as_int(ta) - 0x4B400000) << 23));
  b = __int_as_float(__float_as_int(pb) + ((__float_as_int(tb) - 0x4B400000) << 23));
}

}  // namespace attn
}  // namespace icsa
