// fa8_softmax.cuh — per-row online-softmax step of the FP8 attention kernel.
//
// One thread owns one query row and holds that row's NC scores of the
// current K/V tile in registers (loaded from TMEM). The step:
//   1. row max (three-input max chains),
//   2. warp-uniform lazy-rescale decision: the reference rescales O on every
//      tile (csrc/flash_attention.cu:80-86); here the running max only moves
//      (and O is rescaled) when some row of the warp grew by more than
//      kRescaleThreshold in log2 units,
//   3. p = 2^(s * scale * log2e - (m - kPShift)) for every column. MUFU ex2
//      by default; kEmuPer8 of every 8 columns can instead use a polynomial
//      exp2 on the FMA pipe (range reduction x = n + f with n = round(x) via
//      the 1.5 * 2^23 magic constant, degree-3 polynomial for 2^f on
//      [-0.5, 0.5] fitted by iterated weighted least squares to a relative
//      error of 7.7e-5, then n added to the exponent field with an integer
//      multiply-add),
//   4. row sum of fp32 p (packed f32x2 adds),
//   5. e4m3 requantisation of P (hi) and, for split tiles, of P - hi (lo).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace fa8 {

constexpr float kPShift = 6.0f;            // log2 of the P scale-up
#ifndef FA8_RESCALE_THRESHOLD
#define FA8_RESCALE_THRESHOLD 2.75f  // largest P = 2^(6 + 2.75) = 430
#endif
constexpr float kRescaleThreshold = FA8_RESCALE_THRESHOLD;  // log2 units
static_assert(kPShift + kRescaleThreshold <= 8.8f, "largest P must stay below e4m3's 448");

#ifndef FA8_FUSED_CVT
#define FA8_FUSED_CVT 1
#endif
#ifndef FA8_MAX_TREE
#define FA8_MAX_TREE 1
#endif
#ifndef FA8_EMU_DEG
#define FA8_EMU_DEG 3
#endif
namespace emu {
// 2^f on [-0.5, 0.5]: c0 + f (c1 + f (c2 + f c3)), max relative error 7.7e-5.
constexpr float kC0 = 0.999928891658783f;
constexpr float kC1 = 0.6932758092880249f;
constexpr float kC2 = 0.24260424077510834f;
constexpr float kC3 = 0.05509091913700104f;
// Degree-2 alternative: d0 + f (d1 + f d2), max relative error 1.8e-3 (well
// below e4m3's 2^-4 rounding step of P).
constexpr float kD0 = 1.0005117654800415f;
constexpr float kD1 = 0.7033979296684265f;
constexpr float kD2 = 0.23784694075584412f;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: x + magic rounds x to an integer
constexpr float kClampLo = -30.0f;     // 2^-30 is far below e4m3's smallest subnormal
}  // namespace emu

// Polynomial exp2 of a packed pair (FMA pipe + two integer multiply-adds).
__device__ __forceinline__ uint64_t exp2_emu_pair(float x0, float x1) {
  x0 = fmaxf(x0, emu::kClampLo);
  x1 = fmaxf(x1, emu::kClampLo);
  const uint64_t x = ptx::pack2(x0, x1);
  const uint64_t t = ptx::fadd2(x, ptx::pack2(emu::kMagic, emu::kMagic));
  const uint64_t n = ptx::fadd2(t, ptx::pack2(-emu::kMagic, -emu::kMagic));
  const uint64_t f = ptx::ffma2(n, ptx::pack2(-1.f, -1.f), x);
#if FA8_EMU_DEG == 2
  uint64_t p = ptx::ffma2(ptx::pack2(emu::kD2, emu::kD2), f, ptx::pack2(emu::kD1, emu::kD1));
  p = ptx::ffma2(p, f, ptx::pack2(emu::kD0, emu::kD0));
#else
  uint64_t p = ptx::ffma2(ptx::pack2(emu::kC3, emu::kC3), f, ptx::pack2(emu::kC2, emu::kC2));
  p = ptx::ffma2(p, f, ptx::pack2(emu::kC1, emu::kC1));
  p = ptx::ffma2(p, f, ptx::pack2(emu::kC0, emu::kC0));
#endif
  // bits(t) = bits(magic) + n; (bits(t) << 23) == n << 23 modulo 2^32.
  uint32_t t0, t1, p0, p1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(t0), "=r"(t1) : "l"(t));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(p0), "=r"(p1) : "l"(p));
  uint32_t r0, r1;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(r0) : "r"(t0), "r"(p0));
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(r1) : "r"(t1), "r"(p1));
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(r0), "r"(r1));
  return r;
}

// Result of one softmax step for the owning thread's row.
struct StepOut {
  float alpha;  // factor to apply to the row's O accumulator (1 if !need)
  bool need;    // warp-uniform: O must be rescaled by alpha
#ifdef FA8_TRACE
  long long t_max, t_exp;  // clock64 after the rescale decision / the exp loop
#endif
};

// kFuse (callers that pass split = false): P is converted inside the exp loop.
// kStream (with kFuse): each 16-byte chunk of the e4m3 row is also stored to
// shared memory as soon as it is converted, at p_row + ((chunk ^ swz) << 4)
// (the 128B-swizzled row layout of the PV product's A operand), so the
// stores overlap the rest of the exp loop.
template <int NC, int kEmuPer8, bool kFuse = false, bool kStream = false>
__device__ __forceinline__ StepOut softmax_row_step(float (&s)[NC], float sl2, bool first,
                                                    bool split, float& m_run, float& l_run,
                                                    uint32_t (&ph)[NC / 4],
                                                    uint32_t (&pl)[NC / 4],
                                                    uint32_t p_row = 0, uint32_t swz = 0) {
  static_assert(!kStream || (kFuse && NC == 128), "streamed P stores need the fused loop");
  static_assert(NC % 16 == 0, "row length must be a multiple of 16");
  // 1. row max
#if FA8_MAX_TREE
  // Balanced three-input max tree: the same instruction count as the chains
  // below, dependency depth about log3(NC) instead of NC / 16 + 3.
  float mx;
  {
    float l1[(NC + 2) / 3];
#pragma unroll
    for (int i = 0; i < NC / 3; ++i) l1[i] = ptx::fmax3(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
    constexpr int n1 = NC / 3 + (NC % 3 ? 1 : 0);
    if constexpr (NC % 3 == 1) l1[n1 - 1] = s[NC - 1];
    if constexpr (NC % 3 == 2) l1[n1 - 1] = fmaxf(s[NC - 2], s[NC - 1]);
    int n = n1;
#pragma unroll
    for (int level = 0; level < 6; ++level) {
      if (n <= 1) break;
      const int m = n / 3, rem = n % 3;
#pragma unroll
      for (int i = 0; i < (NC + 2) / 3; ++i)
        if (i < m) l1[i] = ptx::fmax3(l1[3 * i], l1[3 * i + 1], l1[3 * i + 2]);
      if (rem == 1) l1[m] = l1[n - 1];
      if (rem == 2) l1[m] = fmaxf(l1[n - 2], l1[n - 1]);
      n = m + (rem ? 1 : 0);
    }
    mx = l1[0];
  }
#else
  constexpr int G = NC / 16;
  float mxg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float a = ptx::fmax3(s[16 * g + 0], s[16 * g + 1], s[16 * g + 2]);
#pragma unroll
    for (int c = 3; c < 15; c += 2) a = ptx::fmax3(a, s[16 * g + c], s[16 * g + c + 1]);
    mxg[g] = fmaxf(a, s[16 * g + 15]);
  }
  float mx = mxg[0];
#pragma unroll
  for (int g = 1; g < G; ++g) mx = fmaxf(mx, mxg[g]);
#endif

  // 2. lazy rescale decision
  StepOut out;
  const float m_tile = mx * sl2;
  const float m_new = fmaxf(m_run, m_tile);
  out.need = __any_sync(0xffffffffu, m_new > m_run + kRescaleThreshold || first);
  const float m_use = out.need ? m_new : m_run;
  const float base = (m_use == -INFINITY) ? 0.f : (m_use - kPShift);
  out.alpha = 1.f;
  if (out.need) out.alpha = (m_run == -INFINITY) ? 0.f : ptx::ex2(m_run - m_use);
  m_run = m_use;
#ifdef FA8_TRACE
  out.t_max = clock64();
#endif

  // 3 + 4. exponentials and row sum
  const uint64_t sl2x2 = ptx::pack2(sl2, sl2);
  const uint64_t nbx2 = ptx::pack2(-base, -base);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c = 0; c < NC; c += 2) {
    const uint64_t x = ptx::ffma2(ptx::pack2(s[c], s[c + 1]), sl2x2, nbx2);
    float x0, x1;
    ptx::unpack2(x, x0, x1);
    uint64_t e;
    if ((c % 8) < kEmuPer8) {
      e = exp2_emu_pair(x0, x1);
      ptx::unpack2(e, s[c], s[c + 1]);
    } else {
      s[c] = ptx::ex2(x0);
      s[c + 1] = ptx::ex2(x1);
      e = ptx::pack2(s[c], s[c + 1]);
    }
    acc[(c / 2) % 4] = ptx::fadd2(acc[(c / 2) % 4], e);
#if FA8_FUSED_CVT
    // Without the split, each group of four is converted as soon as it is
    // ready, so the e4m3 conversions of earlier columns overlap the ex2 of
    // later ones instead of forming a separate phase.
    if (kFuse && (c % 4) == 2)
      ph[c / 4] = ptx::cvt_e4m3x4(s[c - 2], s[c - 1], s[c], s[c + 1]);
    if (kStream && (c % 16) == 14)
      ptx::st_shared_v4(p_row + (((uint32_t)(c / 16) ^ swz) << 4), ph[c / 4 - 3], ph[c / 4 - 2],
                        ph[c / 4 - 1], ph[c / 4]);
#endif
  }
  {
    const uint64_t a01 = ptx::fadd2(acc[0], acc[1]);
    const uint64_t a23 = ptx::fadd2(acc[2], acc[3]);
    float u0, u1;
    ptx::unpack2(ptx::fadd2(a01, a23), u0, u1);
    l_run = l_run * out.alpha + (u0 + u1);
  }
#ifdef FA8_TRACE
  out.t_exp = clock64();
#endif

  // 5. e4m3 P (hi) and, for split tiles, the e4m3 residual P - hi (lo). Two
  //    separate loops so the common (no split) path carries no branches.
  if (!split) {
#pragma unroll
    for (int j = 0; j < NC / 4; ++j) {
      if (!(FA8_FUSED_CVT && kFuse))
        ph[j] = ptx::cvt_e4m3x4(s[4 * j], s[4 * j + 1], s[4 * j + 2], s[4 * j + 3]);
      pl[j] = 0u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC / 4; ++j) {
      ph[j] = ptx::cvt_e4m3x4(s[4 * j], s[4 * j + 1], s[4 * j + 2], s[4 * j + 3]);
      const uint32_t h01 = ptx::cvt_e4m3x2_to_f16x2((uint16_t)(ph[j] & 0xffffu));
      const uint32_t h23 = ptx::cvt_e4m3x2_to_f16x2((uint16_t)(ph[j] >> 16));
      const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
      const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
      pl[j] = ptx::cvt_e4m3x4(s[4 * j] - f01.x, s[4 * j + 1] - f01.y, s[4 * j + 2] - f23.x,
                              s[4 * j + 3] - f23.y);
    }
  }
  return out;
}

}  // namespace fa8
