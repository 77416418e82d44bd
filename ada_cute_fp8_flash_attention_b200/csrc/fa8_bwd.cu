// fa8_bwd.cu — backward pass of the FP8 attention forward (sm_100a).
//
// The reference has no backward (it exports only the forward,
// csrc/attention_api.cpp:6-9). This computes the gradients of
//   O = softmax(scale * Q K^T, causal mask) V
// for the e4m3 Q/K/V the forward consumed, given dO (fp16), the forward's O
// (fp16) and its natural-log LSE (fp32):
//   P = exp(scale * Q K^T - LSE),  dV = P^T dO,  dP = dO V^T,
//   Delta = rowsum(dO * O),  dS = P * (dP - Delta),
//   dQ = scale * dS K,  dK = scale * dS^T Q.
// P is recomputed exactly in fp32 (not the e4m3 P of the forward).
//
// Three launches:
//   1. bwd_prep_kernel: e4m3 -> fp16 copies of Q, K, V (exact: every e4m3 value
//      is an fp16 value) in the row layout [s][d], sequence padded to a
//      multiple of 128 with zeros. Products that need a tile transposed read
//      the same copy as an MN-major operand.
//   2. bwd_delta_kernel: Delta = rowsum(dO * O) in fp32.
//   3. bwd_tile_kernel<D, false> (dK, dV; one CTA per 128-key tile and KV
//      head): for each query tile, S^T = K Q^T and dP^T = V dO^T into TMEM
//      (tcgen05, f16 x f16 -> f32), turned into fp16 P^T and dS^T in TMEM by
//      16 warps; dV += P^T dO and dK += dS^T Q read A from TMEM and
//      accumulate in TMEM.
//   4. bwd_tile_kernel<D, true> (dQ; one CTA per 128-query tile and head):
//      for each key tile, S = Q K^T, dP = dO V^T, dS in fp16, dQ += dS K.
// Warp-specialised: a TMA warp streams the tiles (double-buffered), one thread
// issues every product, and the streamed tile is split into two 64-column
// halves so that one half's elementwise pass overlaps the other half's
// products. Every wait is bounded and reports a timeout in the status word
// instead of hanging.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "../../include/fa8.h"
#include "sm100_ptx.cuh"

int fa8_note_error(int status, const char* msg);
int fa8_note_cuda_error(cudaError_t e, const char* where);
void fa8_note_launch();

namespace fa8 {
namespace bwd {

constexpr int kTile = 128;                 // query / key rows per tile
constexpr int kPanelBytes = 128 * 128;     // [128 rows][64 halves], 128B swizzled
constexpr long long kTimeout = 4000000000LL;

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for f16 x f16 -> f32, A and B K-major: the same bit
// fields as the e4m3 descriptor (format code 0 is f16 under kind::f16).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return ptx::idesc_e4m3_f32(m, n);
}

// Descriptor of K step kk (16 halves = 32 bytes) of an operand stored as
// 64-column panels of `panel_bytes` each.
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk, int panel_bytes) {
  return ptx::smem_desc_kmajor(base + (uint32_t)((kk >> 2) * panel_bytes + (kk & 3) * 32), 128);
}

// Descriptor of K step kk (16 rows of 128 B) of an MN-major operand stored as
// [K rows][64-column] panels, 128B swizzled as TMA writes a [rows][D] tile:
// 64-column atoms along MN are `lbo` bytes apart (the panel size), 8-row groups
// along K 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int kk, uint32_t lbo) {
  const uint32_t saddr = base + (uint32_t)kk * 2048u;
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct Params {
  int batch, heads, heads_kv, group, sq, skv, sqp, skvp, causal;
  float scale, sl2;         // softmax scale, scale * log2(e)
  const float* lse;         // [b][h][sq] natural log
  const float* delta;       // [b][h][sqp]
  float* dq;                // [b][h][sq][D]
  float* dk;                // [b][hkv][skv][D]
  float* dv;
  int* status;
  long long timeout;
};

// ------------------------------------------------------------------ prep
// out_sd[b][h][sp][D] and/or out_ds[b][h][D][sp] (fp16) from in (e4m3 or fp16)
// addressed in + b*sb + h*sh + s*ss + d*sd; rows s >= S are zero.
template <typename TIn>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const TIn* in, long long sb, long long sh,
                                                       long long ss, long long sd, int H, int S,
                                                       int Sp, int D, __half* out_sd,
                                                       __half* out_ds) {
  __shared__ __half tile[64][65];
  const int bh = blockIdx.z;
  const int b = bh / H, h = bh % H;
  const int s0 = blockIdx.x * 64, d0 = blockIdx.y * 64;
  const TIn* src = in + (long long)b * sb + (long long)h * sh;
  // load 64 x 64 (s, d): consecutive threads walk the input's unit-stride dimension
  const bool d_fast = sd == 1;
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    const int a = i / 64, c = i % 64;
    const int s = d_fast ? s0 + a : s0 + c;
    const int d = d_fast ? d0 + c : d0 + a;
    float v = 0.f;
    if (s < S) {
      const TIn x = src[(long long)s * ss + (long long)d * sd];
      if constexpr (sizeof(TIn) == 1) {
        const __half_raw hr =
            __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(x), __NV_E4M3);
        v = __half2float(__half(hr));
      } else {
        v = __half2float(x);
      }
    }
    tile[s - s0][d - d0] = __float2half_rn(v);
  }
  __syncthreads();
  const long long base_sd = ((long long)b * H + h) * (long long)Sp * D;
  if (out_sd)
    for (int i = threadIdx.x; i < 64 * 64; i += 256) {
      const int a = i / 64, c = i % 64;
      out_sd[base_sd + (long long)(s0 + a) * D + d0 + c] = tile[a][c];
    }
  if (out_ds)
    for (int i = threadIdx.x; i < 64 * 64; i += 256) {
      const int a = i / 64, c = i % 64;
      out_ds[base_sd + (long long)(d0 + a) * Sp + s0 + c] = tile[c][a];
    }
}

// Delta[b][h][s] = sum_d dO * O (fp16 inputs, [b][h][s][D] contiguous); one warp per row.
__global__ void __launch_bounds__(256) bwd_delta_kernel(const __half* d_o, const __half* o,
                                                        float* delta, int H, int S, int Sp, int D,
                                                        long long rows) {
  const long long w = ((long long)blockIdx.x * 256 + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= rows) return;
  const long long bh = w / Sp;
  const int s = (int)(w % Sp);
  float acc = 0.f;
  if (s < S) {
    const __half* a = d_o + (bh * S + s) * D;
    const __half* c = o + (bh * S + s) * D;
    for (int d = lane; d < D; d += 32) acc += __half2float(a[d]) * __half2float(c[d]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[w] = acc;
}

// ------------------------------------------------------------------ shared parts
// Warp-collective store of 16 consecutive 32-bit TMEM columns (one per register).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]: A is M = 128 lanes x K = 16 halves packed two
// per 32-bit column (8 columns).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TMEM column of K step kk of a 128-wide fp16 operand that the elementwise
// pass wrote as 16-column blocks at the start of each 32-column chunk.
__device__ __forceinline__ uint32_t ts_col(int kk) { return 32u * (kk >> 1) + 8u * (kk & 1); }

// ------------------------------------------------------------------ tile kernel
// One kernel body for both passes. A CTA owns a fixed 128-row tile (dK/dV:
// 128 keys of one K/V head; dQ: 128 queries of one head) and streams 128-column
// tiles of the other side (query tiles of every head of the group; key tiles).
// Each streamed tile is handled as two 64-column halves that ping-pong: while
// 8 warps turn half a's S/dP into fp16 P/dS, the tensor pipe runs half b's
// products, and the reverse.
//   warps 0-15  elementwise: half h = w / 8, TMEM lanes 32 (w % 4) .., columns
//               32 ((w / 4) % 2) .. of the half
//   warp 16     TMA producer (lane 0)
//   warp 17     TMEM allocation; lane 0 issues every tcgen05.mma
// TMEM columns: half h: S at 128 h, dP at 128 h + 64 (P, dS written back into
// the first 16 columns of each 32-column chunk); accumulators at 256 (dV or
// dQ) and 256 + D (dK).
constexpr int kWarpsEw = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kThreadsTile = 18 * 32;

template <int D, bool kDq>
struct TileCfg {
  static constexpr int kRowTile = kTile * D * 2;          // [128][D] fp16 (D / 64 panels)
  static constexpr int kOffA = 0;                         // fixed: K (dkdv) or Q (dq)
  static constexpr int kOffA2 = kOffA + kRowTile;         // fixed: V (dkdv) or dO (dq)
  static constexpr int kOffB = kOffA2 + kRowTile;         // streamed: Q / K, two buffers
  static constexpr int kOffB2 = kOffB + 2 * kRowTile;     // streamed: dO / V, two buffers
  static constexpr int kSmem = kOffB2 + 2 * kRowTile;
  static constexpr int kSmemAlloc = kSmem + 1024;
  static constexpr uint32_t kColAcc1 = 256, kColAcc2 = 256 + D;
};

struct TileBars {
  uint64_t fixed_full;
  uint64_t ld_full[2], ld_empty[2];
  uint64_t s_full[2], p_full[2], e_done[2];
  uint64_t acc_done;
};

__device__ __forceinline__ bool wait_bar_abort(uint64_t* bar, uint32_t parity, long long limit,
                                               volatile int* abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

template <int D, bool kDq>
__global__ void __launch_bounds__(kThreadsTile, 1)
    bwd_tile_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const Params p) {
  using C = TileCfg<D, kDq>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ TileBars bars;
  __shared__ uint32_t tmem_sh;
  __shared__ int abort_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = ptx::smem_u32(smem);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  // Fixed tile: blockIdx.x = tile, y = head (K/V head for dK/dV), z = batch.
  // Causal dQ: query tile i streams i + 1 key tiles, so the grid runs the
  // last (heaviest) tiles first; dK/dV's heaviest tiles are already the first.
  const int fx = (kDq && p.causal) ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
  const int hy = blockIdx.y, b = blockIdx.z;
  int n_iter, i_lo = 0;
  if constexpr (kDq) {
    const int nkv = (p.skv + kTile - 1) / kTile;
    n_iter = p.causal ? min(fx + 1, nkv) : nkv;
  } else {
    const int nq = (p.sq + kTile - 1) / kTile;
    i_lo = p.causal ? fx : 0;
    n_iter = (i_lo < nq ? nq - i_lo : 0) * p.group;
  }
  volatile int* abort_flag = &abort_sh;

  if (tid == 0) {
    ptx::mbar_init(&bars.fixed_full, 1);
    for (int x = 0; x < 2; ++x) {
      ptx::mbar_init(&bars.ld_full[x], 1);
      ptx::mbar_init(&bars.ld_empty[x], 1);
      ptx::mbar_init(&bars.s_full[x], 1);
      ptx::mbar_init(&bars.p_full[x], 8);
      ptx::mbar_init(&bars.e_done[x], 1);
    }
    ptx::mbar_init(&bars.acc_done, 1);
    abort_sh = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(&tmem_sh, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_sh;
  bool ok = true;

  // Streamed tile t: (query tile, head) for dK/dV, key tile for dQ.
  auto stream_coords = [&](int t, int& row_tile, int& head) {
    if constexpr (kDq) {
      row_tile = t;
      head = hy / p.group;
    } else {
      row_tile = i_lo + t / p.group;
      head = hy * p.group + t % p.group;
    }
  };

  if (warp == kProducerWarp) {
    if (lane == 0 && n_iter > 0) {
      const uint64_t pol = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(&bars.fixed_full, 2 * C::kRowTile);
#pragma unroll
      for (int pnl = 0; pnl < D / 64; ++pnl) {
        if constexpr (kDq) {
          ptx::tma_load_4d(smem + C::kOffA + pnl * kPanelBytes, &tm_q, &bars.fixed_full, pnl * 64, fx * kTile, hy, b, pol);
          ptx::tma_load_4d(smem + C::kOffA2 + pnl * kPanelBytes, &tm_do, &bars.fixed_full, pnl * 64, fx * kTile, hy, b, pol);
        } else {
          ptx::tma_load_4d(smem + C::kOffA + pnl * kPanelBytes, &tm_k, &bars.fixed_full, pnl * 64, fx * kTile, hy, b, pol);
          ptx::tma_load_4d(smem + C::kOffA2 + pnl * kPanelBytes, &tm_v, &bars.fixed_full, pnl * 64, fx * kTile, hy, b, pol);
        }
      }
      int issued = 0;
      for (int t = 0; t < n_iter; ++t) {
        const int buf = t & 1;
        if (t >= 2 &&
            !wait_bar_abort(&bars.ld_empty[buf], (uint32_t)((t >> 1) - 1) & 1u, p.timeout, abort_flag))
          break;
        int rt, hh;
        stream_coords(t, rt, hh);
        ptx::mbar_arrive_expect_tx(&bars.ld_full[buf], 2 * C::kRowTile);
#pragma unroll
        for (int pnl = 0; pnl < D / 64; ++pnl) {
          uint8_t* d1 = smem + C::kOffB + buf * C::kRowTile + pnl * kPanelBytes;
          uint8_t* d2 = smem + C::kOffB2 + buf * C::kRowTile + pnl * kPanelBytes;
          if constexpr (kDq) {
            ptx::tma_load_4d(d1, &tm_k, &bars.ld_full[buf], pnl * 64, rt * kTile, hh, b, pol);
            ptx::tma_load_4d(d2, &tm_v, &bars.ld_full[buf], pnl * 64, rt * kTile, hh, b, pol);
          } else {
            ptx::tma_load_4d(d1, &tm_q, &bars.ld_full[buf], pnl * 64, rt * kTile, hh, b, pol);
            ptx::tma_load_4d(d2, &tm_do, &bars.ld_full[buf], pnl * 64, rt * kTile, hh, b, pol);
          }
        }
        ++issued;
      }
      // Copies still in flight must land before the CTA exits (bounded waits).
      for (int t = max(0, issued - 2); t < issued; ++t) {
        const long long t0 = clock64();
        while (!ptx::mbar_try_wait(&bars.ld_full[t & 1], (uint32_t)(t >> 1) & 1u) &&
               clock64() - t0 < p.timeout) {
        }
      }
      {
        const long long t0 = clock64();
        while (!ptx::mbar_try_wait(&bars.fixed_full, 0) && clock64() - t0 < p.timeout) {
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && n_iter > 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, 64);
      constexpr uint32_t idesc_e = ptx::idesc_e4m3_f32(128, D, true);  // B MN-major
      const uint32_t a1 = sb + C::kOffA, a2 = sb + C::kOffA2;
      ok = wait_bar_abort(&bars.fixed_full, 0, p.timeout, abort_flag);
      // S_h(t) = A1 B1_h^T, dP_h(t) = A2 B2_h^T (64 columns each)
      auto issue_s = [&](int t, int h) -> bool {
        const int buf = t & 1;
        if (h == 0 && !wait_bar_abort(&bars.ld_full[buf], (uint32_t)(t >> 1) & 1u, p.timeout, abort_flag))
          return false;
        ptx::tc_fence_after();
        const uint32_t b1 = sb + C::kOffB + buf * C::kRowTile + h * 8192;
        const uint32_t b2 = sb + C::kOffB2 + buf * C::kRowTile + h * 8192;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16(tmem + 128 * h, desc_k(a1, kk, kPanelBytes), desc_k(b1, kk, kPanelBytes), idesc_s, kk > 0);
          umma_f16(tmem + 128 * h + 64, desc_k(a2, kk, kPanelBytes), desc_k(b2, kk, kPanelBytes), idesc_s, kk > 0);
        }
        ptx::umma_commit(&bars.s_full[h]);
        return true;
      };
      // Accumulator products of half h of tile t (K = 64 columns of the half).
      auto issue_e = [&](int t, int h) -> bool {
        if (!wait_bar_abort(&bars.p_full[h], (uint32_t)t & 1u, p.timeout, abort_flag)) return false;
        ptx::tc_fence_after();
        const int buf = t & 1;
        const uint32_t b1 = sb + C::kOffB + buf * C::kRowTile;   // Q_t or K_t
        const uint32_t b2 = sb + C::kOffB2 + buf * C::kRowTile;  // dO_t
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (t > 0 || h > 0 || kk > 0) ? 1u : 0u;
          if constexpr (kDq) {
            umma_f16_ts(tmem + C::kColAcc1, tmem + 128 * h + 64 + ts_col(kk),
                        desc_mn(b1, kk + 4 * h, kPanelBytes), idesc_e, acc);
          } else {
            umma_f16_ts(tmem + C::kColAcc1, tmem + 128 * h + ts_col(kk),
                        desc_mn(b2, kk + 4 * h, kPanelBytes), idesc_e, acc);
            umma_f16_ts(tmem + C::kColAcc2, tmem + 128 * h + 64 + ts_col(kk),
                        desc_mn(b1, kk + 4 * h, kPanelBytes), idesc_e, acc);
          }
        }
        ptx::umma_commit(&bars.e_done[h]);
        return true;
      };
      if (ok) ok = issue_s(0, 0) && issue_s(0, 1);
      for (int t = 0; t < n_iter && ok; ++t) {
        ok = issue_e(t, 0);
        if (!ok) break;
        if (t + 1 < n_iter) {
          ok = wait_bar_abort(&bars.e_done[0], (uint32_t)t & 1u, p.timeout, abort_flag) && issue_s(t + 1, 0);
          if (!ok) break;
        }
        ok = issue_e(t, 1);
        if (!ok) break;
        ptx::umma_commit(&bars.ld_empty[t & 1]);
        if (t + 1 < n_iter) {
          ok = wait_bar_abort(&bars.e_done[1], (uint32_t)t & 1u, p.timeout, abort_flag) && issue_s(t + 1, 1);
          if (!ok) break;
        }
      }
      ptx::umma_commit(&bars.acc_done);
      // Drain: every product issued here completes before TMEM is freed.
      const long long t0 = clock64();
      while (!ptx::mbar_try_wait(&bars.acc_done, 0) && clock64() - t0 < p.timeout) {
      }
    }
  } else {
    // ------------------------------------------------------ elementwise warps
    const int h = warp >> 3, quad = warp & 3, chunk = (warp >> 2) & 1;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col_s = 128 * h + 32 * chunk, col_dp = col_s + 64;
    const int row_g = fx * kTile + r;  // key (dK/dV) or query (dQ) of this TMEM lane
    float row_lse2 = INFINITY, row_delta = 0.f;
    if constexpr (kDq) {
      if (row_g < p.sq) {
        const long long rr = (long long)b * p.heads + hy;
        const float l = p.lse[rr * p.sq + row_g];
        row_lse2 = (l == -INFINITY) ? INFINITY : l * 1.4426950408889634f;
        row_delta = p.delta[rr * p.sqp + row_g];
      }
    }
    for (int t = 0; t < n_iter && ok; ++t) {
      int rt, hh;
      stream_coords(t, rt, hh);
      const int c0 = rt * kTile + 64 * h + 32 * chunk;  // first column (query / key) of this warp
      float lse2_l = INFINITY, delta_l = 0.f;             // dK/dV: this lane's column
      if constexpr (!kDq) {
        const int qc = c0 + lane;
        const long long rr = (long long)b * p.heads + hh;
        if (qc < p.sq) {
          const float l = __ldg(p.lse + rr * p.sq + qc);
          lse2_l = (l == -INFINITY) ? INFINITY : l * 1.4426950408889634f;
        }
        delta_l = __ldg(p.delta + rr * p.sqp + qc);
      }
      ok = wait_bar_abort(&bars.s_full[h], (uint32_t)t & 1u, p.timeout, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      ptx::tc_fence_after();
      uint32_t us[32], ud[32];
      ptx::tmem_ld32(tmem + lane_off + col_s, us);
      ptx::tmem_ld32(tmem + lane_off + col_dp, ud);
      ptx::tmem_wait_ld();
      ptx::reg_fence32(us);
      ptx::reg_fence32(ud);
      bool full;
      if constexpr (kDq)
        full = row_g < p.sq && c0 + 31 < p.skv && (!p.causal || c0 + 31 <= row_g);
      else
        full = row_g < p.skv && c0 + 31 < p.sq && (!p.causal || row_g <= c0);
      uint32_t hp[16], hd[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pv[2], dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int col = c0 + e + u;
          float l2, dl;
          bool valid;
          if constexpr (kDq) {
            l2 = row_lse2;
            dl = row_delta;
            valid = full || (col < p.skv && row_g < p.sq && (!p.causal || col <= row_g));
          } else {
            l2 = __shfl_sync(0xffffffffu, lse2_l, e + u);
            dl = __shfl_sync(0xffffffffu, delta_l, e + u);
            valid = full || (row_g < p.skv && col < p.sq && (!p.causal || row_g <= col));
          }
          const float pr = valid ? ptx::ex2(__uint_as_float(us[e + u]) * p.sl2 - l2) : 0.f;
          pv[u] = pr;
          dv[u] = pr * (__uint_as_float(ud[e + u]) - dl);
        }
        hp[e / 2] = pack_h2(pv[0], pv[1]);
        hd[e / 2] = pack_h2(dv[0], dv[1]);
      }
      if constexpr (!kDq) tmem_st16(tmem + lane_off + col_s, hp);
      tmem_st16(tmem + lane_off + col_dp, hd);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars.p_full[h]);
    }
  }

  // Epilogue: the accumulators, 32 columns per warp (warps 0..D/32-1 of each lane quarter).
  if (warp < kWarpsEw) {
    const int quad = warp & 3, c4 = warp >> 2;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int row_g = fx * kTile + quad * 32 + lane;
    if (n_iter > 0) ok = ok && wait_bar_abort(&bars.acc_done, 0, p.timeout, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    ptx::tc_fence_after();
    if (c4 < D / 32) {
      const bool have = ok && n_iter > 0 && !*abort_flag;
      uint32_t u1[32], u2[32];
      ptx::tmem_ld32(tmem + lane_off + C::kColAcc1 + c4 * 32, u1);
      if constexpr (!kDq) ptx::tmem_ld32(tmem + lane_off + C::kColAcc2 + c4 * 32, u2);
      ptx::tmem_wait_ld();
      ptx::reg_fence32(u1);
      if constexpr (!kDq) ptx::reg_fence32(u2);
      if constexpr (kDq) {
        if (row_g < p.sq) {
          float* dst = p.dq + (((long long)b * p.heads + hy) * p.sq + row_g) * D + c4 * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst + e) =
                have ? make_float4(__uint_as_float(u1[e]) * p.scale, __uint_as_float(u1[e + 1]) * p.scale,
                                   __uint_as_float(u1[e + 2]) * p.scale, __uint_as_float(u1[e + 3]) * p.scale)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      } else {
        if (row_g < p.skv) {
          const long long off = (((long long)b * p.heads_kv + hy) * p.skv + row_g) * D + c4 * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            *reinterpret_cast<float4*>(p.dv + off + e) =
                have ? make_float4(__uint_as_float(u1[e]), __uint_as_float(u1[e + 1]),
                                   __uint_as_float(u1[e + 2]), __uint_as_float(u1[e + 3]))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(p.dk + off + e) =
                have ? make_float4(__uint_as_float(u2[e]) * p.scale, __uint_as_float(u2[e + 1]) * p.scale,
                                   __uint_as_float(u2[e + 2]) * p.scale, __uint_as_float(u2[e + 3]) * p.scale)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
    }
  }
  if (tid == 0 && *abort_flag && p.status) atomicOr(p.status, FA8_DEVERR_TIMEOUT);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace bwd
}  // namespace fa8

// ====================================================================== host
namespace {

using namespace fa8::bwd;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// fp16 4-D map over a contiguous [batch][heads][rows][inner] tensor, box
// {64, box_rows}, 128B swizzle.
int map_f16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t heads,
            uint64_t batch, uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return fa8_note_error(FA8_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not found");
  cuuint64_t dims[4] = {inner, rows, heads, batch};
  cuuint64_t strides[3] = {inner * 2, inner * rows * 2, inner * rows * heads * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fa8_note_error(FA8_ERR_ALIGNMENT, "fa8_bwd: tensor map encoding failed");
  return FA8_OK;
}

struct WsLayout {
  int64_t sqp, skvp, q_el, kv_el, off_q, off_k, off_v, off_delta, total;
};

WsLayout ws_layout(const fa8_bwd_params* p) {
  WsLayout w{};
  w.sqp = (p->seqlen_q + 127) / 128 * 128;
  w.skvp = (p->seqlen_kv + 127) / 128 * 128;
  w.q_el = p->batch * p->heads * w.sqp * p->head_dim;
  w.kv_el = p->batch * p->heads_kv * w.skvp * p->head_dim;
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  int64_t o = 0;
  w.off_q = o; o += al(w.q_el * 2);
  w.off_k = o; o += al(w.kv_el * 2);
  w.off_v = o; o += al(w.kv_el * 2);
  w.off_delta = o; o += al(p->batch * p->heads * w.sqp * 4);
  w.total = o;
  return w;
}

int check(const fa8_bwd_params* p) {
  if (!p) return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_bwd: null params");
  if (p->head_dim != 64 && p->head_dim != 128)
    return fa8_note_error(FA8_ERR_UNSUPPORTED, "fa8_bwd: head_dim must be 64 or 128");
  if (p->batch < 0 || p->heads <= 0 || p->heads_kv <= 0 || p->seqlen_q < 0 || p->seqlen_kv < 0 ||
      p->heads % p->heads_kv != 0)
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_bwd: bad sizes (heads % heads_kv != 0?)");
  if (p->v_layout != FA8_V_BHDS && p->v_layout != FA8_V_BHSD)
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_bwd: bad v_layout");
  if (p->batch > 65535 || p->heads > 65535 || p->batch * p->heads > 65535)
    return fa8_note_error(FA8_ERR_UNSUPPORTED, "fa8_bwd: batch x heads above the grid limit");
  return FA8_OK;
}

template <int D>
int launch(const fa8_bwd_params* p, void* ws, cudaStream_t st) {
  const WsLayout w = ws_layout(p);
  char* base = static_cast<char*>(ws);
  __half* qh = reinterpret_cast<__half*>(base + w.off_q);
  __half* kh = reinterpret_cast<__half*>(base + w.off_k);
  __half* vh = reinterpret_cast<__half*>(base + w.off_v);
  float* delta = reinterpret_cast<float*>(base + w.off_delta);
  const int B = (int)p->batch, H = (int)p->heads, Hk = (int)p->heads_kv;
  const int Sq = (int)p->seqlen_q, Skv = (int)p->seqlen_kv;
  const int Sqp = (int)w.sqp, Skvp = (int)w.skvp;
  const long long q_ss = D, q_sh = (long long)Sq * D, q_sb = (long long)H * q_sh;
  const long long k_ss = D, k_sh = (long long)Skv * D, k_sb = (long long)Hk * k_sh;
  // prep
  {
    dim3 gq(Sqp / 64, D / 64, B * H), gk(Skvp / 64, D / 64, B * Hk);
    const uint8_t* q8 = static_cast<const uint8_t*>(p->q);
    const uint8_t* k8 = static_cast<const uint8_t*>(p->k);
    const uint8_t* v8 = static_cast<const uint8_t*>(p->v);
    bwd_prep_kernel<uint8_t><<<gq, 256, 0, st>>>(q8, q_sb, q_sh, q_ss, 1, H, Sq, Sqp, D, qh, nullptr);
    bwd_prep_kernel<uint8_t><<<gk, 256, 0, st>>>(k8, k_sb, k_sh, k_ss, 1, Hk, Skv, Skvp, D, kh, nullptr);
    if (p->v_layout == FA8_V_BHSD)
      bwd_prep_kernel<uint8_t><<<gk, 256, 0, st>>>(v8, k_sb, k_sh, k_ss, 1, Hk, Skv, Skvp, D, vh, nullptr);
    else  // (B, H_kv, D, S_kv): s stride 1, d stride S_kv
      bwd_prep_kernel<uint8_t><<<gk, 256, 0, st>>>(v8, k_sb, k_sh, 1, Skv, Hk, Skv, Skvp, D, vh, nullptr);
    const long long rows = (long long)B * H * Sqp;
    bwd_delta_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(
        static_cast<const __half*>(p->d_o), static_cast<const __half*>(p->o), delta, H, Sq, Sqp, D, rows);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fa8_note_cuda_error(e, "fa8_bwd prep launch");
  }
  CUtensorMap tq, tk, tv, tdo;
  int rc;
  if ((rc = map_f16(&tq, qh, D, Sqp, H, B, 128)) != FA8_OK) return rc;
  if ((rc = map_f16(&tk, kh, D, Skvp, Hk, B, 128)) != FA8_OK) return rc;
  if ((rc = map_f16(&tv, vh, D, Skvp, Hk, B, 128)) != FA8_OK) return rc;
  if ((rc = map_f16(&tdo, p->d_o, D, Sq, H, B, 128)) != FA8_OK) return rc;

  Params kp{};
  kp.batch = B; kp.heads = H; kp.heads_kv = Hk; kp.group = H / Hk;
  kp.sq = Sq; kp.skv = Skv; kp.sqp = Sqp; kp.skvp = Skvp; kp.causal = p->causal ? 1 : 0;
  kp.scale = p->softmax_scale > 0.f ? p->softmax_scale : 1.f / std::sqrt((float)D);
  kp.sl2 = kp.scale * 1.4426950408889634f;
  kp.lse = p->lse; kp.delta = delta;
  kp.dq = p->dq; kp.dk = p->dk; kp.dv = p->dv;
  kp.status = p->status;
  kp.timeout = p->timeout_cycles > 0 ? p->timeout_cycles : kTimeout;

  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fa8_note_error(FA8_ERR_INVALID_ARG, "device index out of range");
  std::call_once(once[dev], [dev] {
    cudaError_t e1 = cudaFuncSetAttribute(bwd_tile_kernel<D, false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          TileCfg<D, false>::kSmemAlloc);
    cudaError_t e2 = cudaFuncSetAttribute(bwd_tile_kernel<D, true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          TileCfg<D, true>::kSmemAlloc);
    attr_err[dev] = e1 != cudaSuccess ? e1 : e2;
  });
  if (attr_err[dev] != cudaSuccess) return fa8_note_cuda_error(attr_err[dev], "cudaFuncSetAttribute (bwd)");
  if (Skv > 0 && B > 0)
    bwd_tile_kernel<D, false><<<dim3(Skvp / 128, Hk, B), kThreadsTile, TileCfg<D, false>::kSmemAlloc, st>>>(
        tq, tk, tv, tdo, kp);
  if (Sq > 0 && B > 0)
    bwd_tile_kernel<D, true><<<dim3(Sqp / 128, H, B), kThreadsTile, TileCfg<D, true>::kSmemAlloc, st>>>(
        tq, tk, tv, tdo, kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fa8_note_cuda_error(e, "fa8_bwd launch");
  fa8_note_launch();
  return FA8_OK;
}

}  // namespace

extern "C" {

void fa8_bwd_params_init(fa8_bwd_params* p, int64_t batch, int64_t heads, int64_t heads_kv,
                         int64_t seqlen_q, int64_t seqlen_kv, int64_t head_dim) {
  if (!p) return;
  *p = fa8_bwd_params{};
  p->batch = batch;
  p->heads = heads;
  p->heads_kv = heads_kv;
  p->seqlen_q = seqlen_q;
  p->seqlen_kv = seqlen_kv;
  p->head_dim = head_dim;
  p->causal = 1;
  p->softmax_scale = 0.f;
  p->v_layout = FA8_V_BHDS;
}

int64_t fa8_bwd_workspace_size(const fa8_bwd_params* p) {
  if (check(p) != FA8_OK) return -1;
  return ws_layout(p).total;
}

int fa8_bwd(const fa8_bwd_params* p, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check(p);
  if (rc != FA8_OK) return rc;
  if (p->batch == 0 || (p->seqlen_q == 0 && p->seqlen_kv == 0)) return FA8_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->seqlen_q == 0 || p->seqlen_kv == 0) {
    // No query sees a key: every gradient is zero (no workspace needed).
    const size_t q_bytes = (size_t)(p->batch * p->heads * p->seqlen_q * p->head_dim) * 4;
    const size_t kv_bytes = (size_t)(p->batch * p->heads_kv * p->seqlen_kv * p->head_dim) * 4;
    if ((q_bytes && !p->dq) || (kv_bytes && (!p->dk || !p->dv)))
      return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_bwd: null gradient pointer");
    cudaError_t e = cudaSuccess;
    if (q_bytes) e = cudaMemsetAsync(p->dq, 0, q_bytes, st);
    if (e == cudaSuccess && kv_bytes) e = cudaMemsetAsync(p->dk, 0, kv_bytes, st);
    if (e == cudaSuccess && kv_bytes) e = cudaMemsetAsync(p->dv, 0, kv_bytes, st);
    return e == cudaSuccess ? FA8_OK : fa8_note_cuda_error(e, "fa8_bwd (empty sequence)");
  }
  if (!p->q || !p->k || !p->v || !p->o || !p->d_o || !p->lse || !p->dq || !p->dk || !p->dv)
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_bwd: null tensor pointer");
  if (!workspace || workspace_bytes < ws_layout(p).total ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fa8_note_error(FA8_ERR_INVALID_ARG,
                          "fa8_bwd: workspace missing, too small (fa8_bwd_workspace_size) or not "
                          "256-byte aligned");
  const void* ptrs16[] = {p->d_o, p->dq, p->dk, p->dv};
  for (const void* q : ptrs16)
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0)
      return fa8_note_error(FA8_ERR_ALIGNMENT, "fa8_bwd: d_o, dq, dk, dv must be 16-byte aligned");
  return p->head_dim == 64 ? launch<64>(p, workspace, st) : launch<128>(p, workspace, st);
}

}  // extern "C"
