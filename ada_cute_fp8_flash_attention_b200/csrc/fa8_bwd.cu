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
//   3. bwd_dkdv_kernel (one CTA per 128-key tile and KV head): for each query
//      tile, S^T = K Q^T and dP^T = V dO^T into TMEM (tcgen05, f16 x f16 -> f32);
//      16 warps (4 per TMEM lane quarter, 32 query columns each) turn them
//      into fp16 P^T and dS^T written back into TMEM; dV += P^T dO and
//      dK += dS^T Q then read A from TMEM and accumulate in TMEM.
//   4. bwd_dq_kernel (one CTA per 128-query tile and head): for each key tile,
//      S = Q K^T and dP = dO V^T, dS in fp16 (TMEM), dQ += dS K in TMEM.
// Operands move by TMA into 128B-swizzled 64-column panels, the next
// iteration's tiles into a second buffer while this one computes; one thread
// issues the tcgen05 products; every wait is bounded and reports a timeout in
// the status word instead of hanging.
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
constexpr int kThreadsBwd = 512;  // 16 warps: warp w reads TMEM lanes 32 (w % 4) .. +31
                                  // and key / query columns 32 (w / 4) .. +31

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

// ------------------------------------------------------------------ dK, dV
template <int D>
struct DkdvCfg {
  static constexpr int kRowTile = kTile * D * 2;     // [128][D] fp16 (D / 64 panels)
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kRowTile;
  static constexpr int kOffQ = kOffV + kRowTile;     // two buffers: Q_i, Q_i+1
  static constexpr int kOffDo = kOffQ + 2 * kRowTile;  // two buffers: dO_i, dO_i+1
  static constexpr int kOffLse = kOffDo + 2 * kRowTile;  // 128 floats: LSE * log2(e)
  static constexpr int kOffDelta = kOffLse + 512;
  static constexpr int kSmem = kOffDelta + 512;
  static constexpr int kSmemAlloc = kSmem + 1024;
  // TMEM: S^T (then P^T) | dP^T (then dS^T) | dV | dK
  static constexpr uint32_t kColS = 0, kColDp = 128, kColDv = 256, kColDk = 256 + D;
};

template <int D>
__global__ void __launch_bounds__(kThreadsBwd, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const Params p) {
  using C = DkdvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_ld[2], bar_mma;
  __shared__ uint32_t tmem_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = ptx::smem_u32(smem);
  float* lse_sh = reinterpret_cast<float*>(smem + C::kOffLse);
  float* delta_sh = reinterpret_cast<float*>(smem + C::kOffDelta);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int quad = warp & 3, chunk = warp >> 2;
  const int r = quad * 32 + lane;  // key row of the tile == TMEM lane
  const int j = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int key = j * kTile + r;
  const int nq = (p.sq + kTile - 1) / kTile;
  const int i_lo = p.causal ? j : 0;
  const int n_heads = p.group;
  const int n_iter = (i_lo < nq ? nq - i_lo : 0) * n_heads;

  if (tid == 0) {
    ptx::mbar_init(&bar_ld[0], 1);
    ptx::mbar_init(&bar_ld[1], 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&tmem_sh, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
  constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);
  constexpr uint32_t idesc_g = ptx::idesc_e4m3_f32(128, D, true);  // B MN-major
  uint32_t ph_mma = 0;
  bool ok = true;

  // Q_i and dO_i of iteration `it` into buffer it & 1 (K_j, V_j with the first).
  auto issue_loads = [&](int it) {
    const int i = i_lo + it / n_heads;
    const int h = hk * p.group + it % n_heads;
    const int buf = it & 1;
    uint32_t bytes = 2 * C::kRowTile;
    if (it == 0) bytes += 2 * C::kRowTile;
    ptx::mbar_arrive_expect_tx(&bar_ld[buf], bytes);
    const uint64_t pol = ptx::policy_evict_last();
#pragma unroll
    for (int pnl = 0; pnl < D / 64; ++pnl) {
      if (it == 0) {
        ptx::tma_load_4d(smem + C::kOffK + pnl * kPanelBytes, &tm_k, &bar_ld[buf], pnl * 64, j * kTile, hk, b, pol);
        ptx::tma_load_4d(smem + C::kOffV + pnl * kPanelBytes, &tm_v, &bar_ld[buf], pnl * 64, j * kTile, hk, b, pol);
      }
      ptx::tma_load_4d(smem + C::kOffQ + buf * C::kRowTile + pnl * kPanelBytes, &tm_q, &bar_ld[buf],
                       pnl * 64, i * kTile, h, b, pol);
      ptx::tma_load_4d(smem + C::kOffDo + buf * C::kRowTile + pnl * kPanelBytes, &tm_do, &bar_ld[buf],
                       pnl * 64, i * kTile, h, b, pol);
    }
  };
  if (tid == 0 && n_iter > 0) issue_loads(0);

  for (int it = 0; it < n_iter && ok; ++it) {
    const int i = i_lo + it / n_heads;
    const int h = hk * p.group + it % n_heads;
    const int buf = it & 1;
    // The other buffer was last read by the products of iteration it - 1 (complete).
    if (tid == 0 && it + 1 < n_iter) issue_loads(it + 1);
    if (tid < kTile) {
      const int q = i * kTile + tid;
      const long long row = ((long long)b * p.heads + h);
      const float l = q < p.sq ? p.lse[row * p.sq + q] : INFINITY;
      lse_sh[tid] = (l == -INFINITY) ? INFINITY : l * 1.4426950408889634f;
      delta_sh[tid] = p.delta[row * p.sqp + i * kTile + tid];
    }
    ok = wait_bar(&bar_ld[buf], (uint32_t)(it >> 1) & 1u, p.timeout);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const uint32_t q_addr = sb + C::kOffQ + buf * C::kRowTile;
    const uint32_t do_addr = sb + C::kOffDo + buf * C::kRowTile;
    // S^T = K Q^T, dP^T = V dO^T
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        umma_f16(tmem + C::kColS, desc_k(sb + C::kOffK, kk, kPanelBytes),
                 desc_k(q_addr, kk, kPanelBytes), idesc_s, kk > 0);
        umma_f16(tmem + C::kColDp, desc_k(sb + C::kOffV, kk, kPanelBytes),
                 desc_k(do_addr, kk, kPanelBytes), idesc_s, kk > 0);
      }
      ptx::umma_commit(&bar_mma);
    }
    ok = wait_bar(&bar_mma, ph_mma, p.timeout);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    // P^T and dS^T of this warp's 32 queries, fp16, back into the first 16
    // columns of the chunk they were read from.
    ptx::tc_fence_after();
    {
      uint32_t us[32], ud[32];
      ptx::tmem_ld32(tmem + lane_off + C::kColS + chunk * 32, us);
      ptx::tmem_ld32(tmem + lane_off + C::kColDp + chunk * 32, ud);
      ptx::tmem_wait_ld();
      ptx::reg_fence32(us);
      ptx::reg_fence32(ud);
      const int q0 = i * kTile + chunk * 32;
      const bool full = key < p.skv && q0 + 31 < p.sq && (!p.causal || key <= q0);
      uint32_t hp[16], hd[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pv[2], dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int qc = chunk * 32 + e + u;
          const int q = q0 + e + u;
          const bool valid = full || (key < p.skv && q < p.sq && (!p.causal || key <= q));
          const float pr = valid ? ptx::ex2(__uint_as_float(us[e + u]) * p.sl2 - lse_sh[qc]) : 0.f;
          pv[u] = pr;
          dv[u] = pr * (__uint_as_float(ud[e + u]) - delta_sh[qc]);
        }
        hp[e / 2] = pack_h2(pv[0], pv[1]);
        hd[e / 2] = pack_h2(dv[0], dv[1]);
      }
      tmem_st16(tmem + lane_off + C::kColS + chunk * 32, hp);
      tmem_st16(tmem + lane_off + C::kColDp + chunk * 32, hd);
      ptx::tmem_wait_st();
    }
    ptx::tc_fence_before();
    ok = __syncthreads_and(ok);
    if (!ok) break;
    // dV += P^T dO, dK += dS^T Q (K = the 128 queries of the tile)
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        umma_f16_ts(tmem + C::kColDv, tmem + C::kColS + ts_col(kk),
                    desc_mn(do_addr, kk, kPanelBytes), idesc_g, (it > 0 || kk > 0));
        umma_f16_ts(tmem + C::kColDk, tmem + C::kColDp + ts_col(kk),
                    desc_mn(q_addr, kk, kPanelBytes), idesc_g, (it > 0 || kk > 0));
      }
      ptx::umma_commit(&bar_mma);
    }
    ok = wait_bar(&bar_mma, ph_mma, p.timeout);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
  }
  if (!ok && tid == 0) {
    if (p.status) atomicOr(p.status, FA8_DEVERR_TIMEOUT);
    // Let copies and products in flight finish (bounded) before TMEM is freed.
    wait_bar(&bar_ld[0], 0, p.timeout);
    wait_bar(&bar_mma, ph_mma, p.timeout);
  }
  __syncthreads();
  // Epilogue: dV and scale * dK rows of this key tile (zero when no query sees them).
  ptx::tc_fence_after();
  if (chunk < D / 32) {
    const bool have = ok && n_iter > 0;
    const long long row_off = (((long long)b * p.heads_kv + hk) * p.skv + key) * D + chunk * 32;
    uint32_t uv[32], uk[32];
    ptx::tmem_ld32(tmem + lane_off + C::kColDv + chunk * 32, uv);
    ptx::tmem_ld32(tmem + lane_off + C::kColDk + chunk * 32, uk);
    ptx::tmem_wait_ld();
    ptx::reg_fence32(uv);
    ptx::reg_fence32(uk);
    if (key < p.skv) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 a = have ? make_float4(__uint_as_float(uv[e]), __uint_as_float(uv[e + 1]),
                                            __uint_as_float(uv[e + 2]), __uint_as_float(uv[e + 3]))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 k4 =
            have ? make_float4(__uint_as_float(uk[e]) * p.scale, __uint_as_float(uk[e + 1]) * p.scale,
                               __uint_as_float(uk[e + 2]) * p.scale, __uint_as_float(uk[e + 3]) * p.scale)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(p.dv + row_off + e) = a;
        *reinterpret_cast<float4*>(p.dk + row_off + e) = k4;
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ dQ
template <int D>
struct DqCfg {
  static constexpr int kRowTile = kTile * D * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffDo = kOffQ + kRowTile;
  static constexpr int kOffK = kOffDo + kRowTile;    // two buffers: K_j, K_j+1
  static constexpr int kOffV = kOffK + 2 * kRowTile;  // two buffers: V_j, V_j+1
  static constexpr int kSmem = kOffV + 2 * kRowTile;
  static constexpr int kSmemAlloc = kSmem + 1024;
  // TMEM: S | dP (then dS) | dQ
  static constexpr uint32_t kColS = 0, kColDp = 128, kColDq = 256;
};

template <int D>
__global__ void __launch_bounds__(kThreadsBwd, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const Params p) {
  using C = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_ld[2], bar_mma;
  __shared__ uint32_t tmem_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = ptx::smem_u32(smem);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int quad = warp & 3, chunk = warp >> 2;
  const int r = quad * 32 + lane;  // query row of the tile == TMEM lane
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int q = i * kTile + r;
  const int nkv = (p.skv + kTile - 1) / kTile;
  const int n_iter = p.causal ? min(i + 1, nkv) : nkv;
  const long long row = (long long)b * p.heads + h;
  float lse2 = INFINITY, delta = 0.f;
  if (q < p.sq) {
    const float l = p.lse[row * p.sq + q];
    lse2 = (l == -INFINITY) ? INFINITY : l * 1.4426950408889634f;
    delta = p.delta[row * p.sqp + q];
  }

  if (tid == 0) {
    ptx::mbar_init(&bar_ld[0], 1);
    ptx::mbar_init(&bar_ld[1], 1);
    ptx::mbar_init(&bar_mma, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&tmem_sh, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
  constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);
  constexpr uint32_t idesc_g = ptx::idesc_e4m3_f32(128, D, true);  // B MN-major
  uint32_t ph_mma = 0;
  bool ok = true;

  auto issue_loads = [&](int jj) {
    const int buf = jj & 1;
    uint32_t bytes = 2 * C::kRowTile;
    if (jj == 0) bytes += 2 * C::kRowTile;
    ptx::mbar_arrive_expect_tx(&bar_ld[buf], bytes);
    const uint64_t pol = ptx::policy_evict_last();
#pragma unroll
    for (int pnl = 0; pnl < D / 64; ++pnl) {
      if (jj == 0) {
        ptx::tma_load_4d(smem + C::kOffQ + pnl * kPanelBytes, &tm_q, &bar_ld[buf], pnl * 64, i * kTile, h, b, pol);
        ptx::tma_load_4d(smem + C::kOffDo + pnl * kPanelBytes, &tm_do, &bar_ld[buf], pnl * 64, i * kTile, h, b, pol);
      }
      ptx::tma_load_4d(smem + C::kOffK + buf * C::kRowTile + pnl * kPanelBytes, &tm_k, &bar_ld[buf],
                       pnl * 64, jj * kTile, hk, b, pol);
      ptx::tma_load_4d(smem + C::kOffV + buf * C::kRowTile + pnl * kPanelBytes, &tm_v, &bar_ld[buf],
                       pnl * 64, jj * kTile, hk, b, pol);
    }
  };
  if (tid == 0 && n_iter > 0) issue_loads(0);

  for (int j = 0; j < n_iter && ok; ++j) {
    const int buf = j & 1;
    if (tid == 0 && j + 1 < n_iter) issue_loads(j + 1);
    ok = wait_bar(&bar_ld[buf], (uint32_t)(j >> 1) & 1u, p.timeout);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const uint32_t k_addr = sb + C::kOffK + buf * C::kRowTile;
    const uint32_t v_addr = sb + C::kOffV + buf * C::kRowTile;
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        umma_f16(tmem + C::kColS, desc_k(sb + C::kOffQ, kk, kPanelBytes),
                 desc_k(k_addr, kk, kPanelBytes), idesc_s, kk > 0);
        umma_f16(tmem + C::kColDp, desc_k(sb + C::kOffDo, kk, kPanelBytes),
                 desc_k(v_addr, kk, kPanelBytes), idesc_s, kk > 0);
      }
      ptx::umma_commit(&bar_mma);
    }
    ok = wait_bar(&bar_mma, ph_mma, p.timeout);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    ptx::tc_fence_after();
    {
      uint32_t us[32], ud[32];
      ptx::tmem_ld32(tmem + lane_off + C::kColS + chunk * 32, us);
      ptx::tmem_ld32(tmem + lane_off + C::kColDp + chunk * 32, ud);
      ptx::tmem_wait_ld();
      ptx::reg_fence32(us);
      ptx::reg_fence32(ud);
      const int k0 = j * kTile + chunk * 32;
      const bool full = q < p.sq && k0 + 31 < p.skv && (!p.causal || k0 + 31 <= q);
      uint32_t hd[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int key = k0 + e + u;
          const bool valid = full || (key < p.skv && q < p.sq && (!p.causal || key <= q));
          const float pr = valid ? ptx::ex2(__uint_as_float(us[e + u]) * p.sl2 - lse2) : 0.f;
          dv[u] = pr * (__uint_as_float(ud[e + u]) - delta);
        }
        hd[e / 2] = pack_h2(dv[0], dv[1]);
      }
      tmem_st16(tmem + lane_off + C::kColDp + chunk * 32, hd);
      ptx::tmem_wait_st();
    }
    ptx::tc_fence_before();
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk)
        umma_f16_ts(tmem + C::kColDq, tmem + C::kColDp + ts_col(kk),
                    desc_mn(k_addr, kk, kPanelBytes), idesc_g, (j > 0 || kk > 0));
      ptx::umma_commit(&bar_mma);
    }
    ok = wait_bar(&bar_mma, ph_mma, p.timeout);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
  }
  if (!ok && tid == 0) {
    if (p.status) atomicOr(p.status, FA8_DEVERR_TIMEOUT);
    wait_bar(&bar_ld[0], 0, p.timeout);
    wait_bar(&bar_mma, ph_mma, p.timeout);
  }
  __syncthreads();
  ptx::tc_fence_after();
  if (chunk < D / 32) {
    const bool have = ok && n_iter > 0;
    uint32_t u[32];
    ptx::tmem_ld32(tmem + lane_off + C::kColDq + chunk * 32, u);
    ptx::tmem_wait_ld();
    ptx::reg_fence32(u);
    if (q < p.sq) {
      float* dst = p.dq + (row * p.sq + q) * D + chunk * 32;
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4*>(dst + e) =
            have ? make_float4(__uint_as_float(u[e]) * p.scale, __uint_as_float(u[e + 1]) * p.scale,
                               __uint_as_float(u[e + 2]) * p.scale, __uint_as_float(u[e + 3]) * p.scale)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
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
  if (p->batch > 65535 || p->heads > 65535)
    return fa8_note_error(FA8_ERR_UNSUPPORTED, "fa8_bwd: batch / heads above the grid limit");
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
    cudaError_t e1 = cudaFuncSetAttribute(bwd_dkdv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          DkdvCfg<D>::kSmemAlloc);
    cudaError_t e2 = cudaFuncSetAttribute(bwd_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          DqCfg<D>::kSmemAlloc);
    attr_err[dev] = e1 != cudaSuccess ? e1 : e2;
  });
  if (attr_err[dev] != cudaSuccess) return fa8_note_cuda_error(attr_err[dev], "cudaFuncSetAttribute (bwd)");
  if (Skv > 0 && B > 0)
    bwd_dkdv_kernel<D><<<dim3(Skvp / 128, Hk, B), kThreadsBwd, DkdvCfg<D>::kSmemAlloc, st>>>(tq, tk, tv, tdo, kp);
  if (Sq > 0 && B > 0)
    bwd_dq_kernel<D><<<dim3(Sqp / 128, H, B), kThreadsBwd, DqCfg<D>::kSmemAlloc, st>>>(tq, tk, tv, tdo, kp);
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return p->head_dim == 64 ? launch<64>(p, workspace, st) : launch<128>(p, workspace, st);
}

}  // extern "C"
