// fa8_fwd_kernel.cuh — warp-specialised FP8 (e4m3) flash-attention forward
// for sm_100a.
//
// Replaces the reference's FA2-style Ada kernel flash_attn_fp8_kernel
// (csrc/flash_attention.cu:90-460) and its traits (csrc/kernel_traits.h:11-87)
// with a Blackwell design:
//
//   * a CTA owns T = 1 (default; two CTAs per SM) or T = 2 (one CTA per SM)
//     128-row query tiles of one (batch, head); 128 (T + 1) threads: T softmax
//     warpgroups and one control warpgroup; setmaxnreg gives the softmax
//     warpgroups 192 (T = 1) or 200 (T = 2) registers per thread;
//   * control warp 1 (TMA) streams K and V tiles (128 keys each) into a ring of
//     shared-memory stages (cp.async.bulk.tensor, mbarrier completion);
//   * control warps 0 and 2 (one elected thread each, one per query tile)
//     issue tcgen05.mma kind::f8f6f4:
//       S_i = Q_i K^T  into TMEM (128 lanes x 128 f32 columns per tile),
//       O_i += P_i V   into TMEM (128 lanes x D f32 columns per tile);
//     K/V tiles are loaded in exactly the order these products use them
//     (K0, K1, V0, K2, V1, ...), so every ring stage is reused first-in
//     first-out;
//   * warps 0-3 (and 4-7) are the softmax warpgroups of Q0 (and Q1). Each thread
//     owns one query row (one TMEM lane): row max and row sum need no
//     shuffles. They run the online softmax in base 2 (the reference's
//     softmax_rescale_o, csrc/flash_attention.cu:54-88, with the scale fixed
//     to softmax_scale * log2(e)), requantise P to e4m3 into a 128B-swizzled
//     shared tile for the PV product (D = 64 with T = 1: into spare TMEM
//     columns, read by the PV product from TMEM), rescale O in TMEM only when the row max
//     grew by more than kRescaleThreshold (lazy rescale), and finally
//     normalise O by the row sum (the reference's final_softmax_rescale_o,
//     csrc/flash_attention.cu:38-52) and store it.
//
// K/V tiles are visited from the last needed tile down to tile 0 — the same
// diagonal-first order as the reference's main loop
// (csrc/flash_attention.cu:345-428) — so for causal attention the masked
// diagonal tile comes first. The causal mask keeps key_pos <= query_pos as
// in csrc/flash_attention.cu:292-304 (and test.py:10-12), in global
// positions (q_offset / kv_offset) so context-parallel chunks mask
// correctly.
//
// Numerics of the P requantisation (the reference casts P in (0,1] straight
// to e4m3, csrc/flash_attention.cu:312-320):
//   * P is formed as 2^(s*scale*log2e - m + kPShift) so typical
//     probabilities sit in e4m3's normal range, not in its subnormals;
//     with the lazy-rescale threshold the largest P is 2^(kPShift +
//     kRescaleThreshold) = 2^8.75 = 430 < 448 (e4m3 max).
//   * for query tiles whose rows see few keys (short causal prefixes) P is
//     split as hi = e4m3(P), lo = e4m3(P - hi) and both are multiplied by V,
//     which brings the relative error of P from 2^-4 to about 2^-8.
//   * the row sum is accumulated from the unquantised fp32 P.
//
// Every mbarrier wait is bounded: after p.timeout_cycles the waiting thread
// raises a CTA-wide abort flag, ORs FA8_DEVERR_TIMEOUT into the optional
// status word and all roles leave their loops, drain their in-flight
// copies / MMAs with bounded waits, free TMEM and exit.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "fa8_softmax.cuh"
#include "sm100_ptx.cuh"

namespace fa8 {

constexpr int kBlockM = 128;           // query rows per tile (= TMEM lanes)
constexpr int kBlockN = 128;           // keys per K/V tile
// A CTA owns T query tiles (T = 2: one CTA per SM; T = 1: two CTAs per SM,
// whose prologues / epilogues overlap each other's main loops). Warps 0..4T-1
// are the softmax warpgroups; the control warpgroup follows: its warp 0
// issues tile 0's MMAs, warp 1 is the TMA producer, warp 2 issues tile 1's.
template <int T>
struct Roles {
  static_assert(T == 1 || T == 2, "one or two query tiles per CTA");
  static constexpr int kThreads = 128 * (T + 1);
  static constexpr int kCtrl = 4 * T;
  static constexpr int kMmaWarp = kCtrl;
  static constexpr int kLoadWarp = kCtrl + 1;
  static constexpr int kMmaWarp2 = kCtrl + 2;
  static constexpr int kMinBlocks = (T == 1) ? 2 : 1;
  // setmaxnreg budgets: control + softmax registers must fit the launch budget
  // (65536 / kMinBlocks per CTA), and per scheduler 2 softmax warps + 1
  // control warp (x kMinBlocks CTAs) must fit its 512 registers per lane.
  static constexpr int kRegsControl = (T == 1) ? 64 : 104;
  static constexpr int kRegsSoftmax = (T == 1) ? 192 : 200;
  static_assert(128 * kRegsControl + 128 * T * kRegsSoftmax <=
                    (65536 / kMinBlocks / (128 * (T + 1))) / 8 * 8 * 128 * (T + 1),
                "setmaxnreg split exceeds the launch register budget");
};
#ifndef FA8_EMU
#define FA8_EMU 2
#endif
// Columns of every 8 whose exp2 runs on the FMA pipe instead of MUFU. Measured
// on B200 (C2 shape, one tile per CTA): 0 -> 1292 TFLOPS, 1 or 2 -> 1339,
// 3 -> 1256; a degree-2 polynomial was no faster than degree 3.
constexpr int kEmuPer8 = FA8_EMU;
#ifndef FA8_STAGGER
#define FA8_STAGGER 1
#endif
constexpr bool kStagger = FA8_STAGGER != 0;
#ifndef FA8_REGS_CONTROL
#define FA8_REGS_CONTROL 1  // 0 = no register reallocation between roles
#endif
#ifndef FA8_TMA_STORE
#define FA8_TMA_STORE 1
#endif
constexpr bool kTmaStore = FA8_TMA_STORE != 0;  // fp16 O tiles leave through TMA stores
#ifndef FA8_P_TMEM
#define FA8_P_TMEM 1
#endif
#ifndef FA8_WAIT_SLEEP
#define FA8_WAIT_SLEEP 20000  // suspend-time hint (ns) of mbarrier waits; 0 = spin
#endif
constexpr long long kTimeoutCycles = 4000000000LL;
constexpr int kDefaultSplitKeys = 1024;

template <int D, int T>
struct TileCfg {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr int kQKRowBytes = D;                  // e4m3 rows of Q and K
  static constexpr int kQBytes = kBlockM * D;
  static constexpr int kKBytes = kBlockN * D;
  static constexpr int kVBytes = D * kBlockN;            // V^T tile: D rows of 128 keys
  static constexpr int kStageBytes = kKBytes;            // == kVBytes
  static constexpr int kStages = (T == 2) ? ((D == 128) ? 6 : 8) : ((D == 128) ? 3 : 8);
  static constexpr int kPBytes = kBlockM * kBlockN;      // 128 rows x 128 B
  static constexpr int kOffQ = 0;
  static constexpr int kOffRing = T * kQBytes;
  static constexpr int kOffP = kOffRing + kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffP + 2 * T * kPBytes;  // hi + lo per tile
  static constexpr int kSmemAlloc = kSmemBytes + 1024;   // slack for 1024-B alignment
  // TMEM columns: S0 | S1 | O0 | O1 (T = 2) or S0 | O0 (T = 1)
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColO = T * kBlockN;
  static constexpr uint32_t kTmemCols = (T == 2) ? 512 : 256;
  // With one tile per CTA and D = 64, 64 TMEM columns are spare: P (hi, lo)
  // lives there (32 columns each) and the PV product reads A from TMEM.
  static constexpr bool kPInTmem = FA8_P_TMEM && T == 1 && D == 64;
  static constexpr uint32_t kColP = kColO + D;
  static constexpr uint32_t kIdescS = ptx::idesc_e4m3_f32(kBlockM, kBlockN);
  static constexpr uint32_t kIdescO = ptx::idesc_e4m3_f32(kBlockM, D);
};

struct KernelParams {
  int batch, heads, heads_kv, seqlen_q, seqlen_kv, head_group;
  int causal, out_e4m3, split_keys, n_qblocks;
  float scale_log2;  // softmax scale x descale_q x descale_k x log2(e)
  float o_scale;     // descale_v
  long long q_offset, kv_offset;
  void* o;
  long long o_sb, o_sh, o_ss;
  float* lse;
  long long lse_sb, lse_sh;
  int* status;
  const int* cu_seqlens_q;   // varlen: (batch + 1) prefix sums, or null
  const int* cu_seqlens_kv;
  int o_tma;                 // tm_o describes O (fp16, 16-byte aligned strides)
  long long timeout_cycles;  // bound of every barrier wait
  int debug_skip_kv_loads;   // test hook: issue no K/V loads (waits run out)
  const float* dq_bh;        // optional per-(batch, head) dequant factors
  const float* dk_bh;
  const float* dv_bh;
  long long dq_sb, dq_sh, dkv_sb, dkv_sh;
};

#ifdef FA8_TRACE
// Debug-only phase timestamps (clock64) of CTA (0,0,0): [role][step][event].
// role 0/1 = softmax warpgroup 0/1 (thread 0 of the group), role 2 = MMA thread.
__device__ long long fa8_trace_buf[3][64][8];
// [slot]: waits that did not succeed on the first probe; [64 + slot]: polls.
__device__ unsigned long long fa8_trace_spin[128];
// Per-CTA (linear block id < 4096): globaltimer at entry and exit, SM id.
__device__ long long fa8_trace_cta[4096][3];
__device__ __forceinline__ long long fa8_gtimer() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define FA8_TR(role, step, ev)                                                 \
  do {                                                                         \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (step) < 64)  \
      fa8_trace_buf[role][step][ev] = clock64();                               \
  } while (0)
#else
#define FA8_TR(role, step, ev) \
  do {                         \
  } while (0)
#endif

// Barrier slots in static shared memory.
template <int NS, int kTilesPerCta>
struct Bars {
  uint64_t q_full[kTilesPerCta];
  uint64_t kv_full[NS];
  uint64_t kv_empty[NS];
  uint64_t s_full[kTilesPerCta];
  uint64_t s_free[kTilesPerCta];
  uint64_t p_full[kTilesPerCta];
  uint64_t o_done[kTilesPerCta];
  uint64_t drain[kTilesPerCta];
  uint64_t offset;  // softmax warpgroup 0 -> 1: first exp phase finished
};

// Bounded wait on phase `parity` of `bar`. Returns false on abort/timeout.
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int* status,
                                             long long limit) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
#ifdef FA8_TRACE
  // Debug: count polls per barrier slot (CTA 0 only).
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
    extern __shared__ uint8_t smem_raw[];
    (void)smem_raw;
    atomicAdd(&fa8_trace_spin[(ptx::smem_u32(bar) & 0x3ff) / 8], 1ull);
  }
#endif
  while (true) {
#ifdef FA8_TRACE
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
      atomicAdd(&fa8_trace_spin[64 + (ptx::smem_u32(bar) & 0x3ff) / 8], 1ull);
#endif
#if FA8_WAIT_SLEEP
    // Suspends until the phase completes (or the hint expires): a waiting warp
    // takes no issue slots from the warps that share its scheduler.
    if (ptx::mbar_try_wait_sleep(bar, parity, FA8_WAIT_SLEEP)) return true;
#else
#pragma unroll 1
    for (int spin = 0; spin < 64; ++spin)
      if (ptx::mbar_try_wait(bar, parity)) return true;
#endif
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      if (status) atomicOr(status, 1);
      return false;
    }
  }
}

// Position of K(t) / V(t) (t-th K/V tile processed, of n) in the load order
// K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1) — the order in which the
// MMA issuer uses them (QK(t+1) is issued before PV(t)).
__device__ __forceinline__ int load_slot_k(int t) { return t == 0 ? 0 : 2 * t - 1; }
__device__ __forceinline__ int load_slot_v(int t, int n) {
  return t == n - 1 ? 2 * n - 1 : 2 * t + 2;
}
__device__ __forceinline__ void load_slot_inverse(int L, int n, bool& is_v, int& t) {
  if (L == 0) {
    is_v = false;
    t = 0;
  } else if (L == 2 * n - 1) {
    is_v = true;
    t = n - 1;
  } else if (L & 1) {
    is_v = false;
    t = (L + 1) / 2;
  } else {
    is_v = true;
    t = (L - 2) / 2;
  }
}

// Number of K/V tiles query tile `i` needs, and whether its P is split.
struct TilePlan {
  int n;       // K/V tiles (tile indices 0 .. n-1)
  int split;   // hi/lo requantisation of P
  int q_start; // first query row (local)
};

template <int kTilesPerCta>
__device__ __forceinline__ TilePlan plan_tile(const KernelParams& p, int qb, int i, int sq,
                                              int skv) {
  TilePlan t;
  t.q_start = qb * (kTilesPerCta * kBlockM) + i * kBlockM;
  t.n = 0;
  t.split = 0;
  if (t.q_start >= sq) return t;
  const int n_kv = (skv + kBlockN - 1) / kBlockN;
  long long visible_first;
  if (p.causal) {
    const long long last_row = min(t.q_start + kBlockM - 1, sq - 1);
    const long long max_key = p.q_offset + last_row - p.kv_offset;  // local key index
    t.n = max_key < 0 ? 0 : (int)min((long long)n_kv, max_key / kBlockN + 1);
    visible_first = p.q_offset + t.q_start - p.kv_offset + 1;
    if (visible_first > skv) visible_first = skv;
  } else {
    t.n = n_kv;
    visible_first = skv;
  }
  t.split = (t.n > 0 && visible_first < p.split_keys) ? 1 : 0;
  return t;
}

// Write one row of O (fp16 or e4m3) from 32 f32 values at column chunk `c`.
__device__ __forceinline__ void store_o_chunk(const KernelParams& p, char* row_ptr, int c,
                                              const float (&v)[32]) {
  if (!p.out_e4m3) {
    uint4* dst = reinterpret_cast<uint4*>(row_ptr + c * 32 * 2);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __half2 h = __floats2half2_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t*>(&h);
      }
      dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    uint4* dst = reinterpret_cast<uint4*>(row_ptr + c * 32);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int base = 16 * j + 4 * e;
        w[e] = (uint32_t)ptx::cvt_e4m3x2(v[base], v[base + 1]) |
               ((uint32_t)ptx::cvt_e4m3x2(v[base + 2], v[base + 3]) << 16);
      }
      dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <int D, int kTilesPerCta>
__global__ void __launch_bounds__(Roles<kTilesPerCta>::kThreads, Roles<kTilesPerCta>::kMinBlocks)
    fa8_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ CUtensorMap tm_o, const KernelParams p) {
  using C = TileCfg<D, kTilesPerCta>;
  using R = Roles<kTilesPerCta>;
  constexpr int kMmaWarp = R::kMmaWarp;
  constexpr int kLoadWarp = R::kLoadWarp;
  constexpr int kMmaWarp2 = R::kMmaWarp2;
  constexpr int kSoftmaxWarps = 4 * kTilesPerCta;
  constexpr bool kStaggerT = kStagger && kTilesPerCta == 2;
  constexpr int NS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars<NS, kTilesPerCta> bars;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
#ifdef FA8_TRACE
  const int cta_lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (threadIdx.x == 0 && cta_lin < 4096) {
    unsigned smid;
    asm volatile("mov.u32 %0, %smid;" : "=r"(smid));
    fa8_trace_cta[cta_lin][0] = fa8_gtimer();
    fa8_trace_cta[cta_lin][2] = smid;
  }
#endif
  if (threadIdx.x == 0) FA8_TR(2, 63, 0);
  const int qb = p.causal ? (p.n_qblocks - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / p.head_group;
  // Variable-length batches: sequence b occupies rows [cu[b], cu[b+1]) of the
  // packed Q / O (and K / V^T) tensors; the TMA batch coordinate is then 0.
  int sq = p.seqlen_q, skv = p.seqlen_kv, q_base = 0, kv_base = 0, tb = b;
  if (p.cu_seqlens_q) {
    q_base = p.cu_seqlens_q[b];
    sq = p.cu_seqlens_q[b + 1] - q_base;
    kv_base = p.cu_seqlens_kv[b];
    skv = p.cu_seqlens_kv[b + 1] - kv_base;
    tb = 0;
    if ((kv_base & 15) != 0 || sq < 0 || skv < 0) {
      // A V^T tile must start on a 16-byte boundary (TMA): refuse the sequence.
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, 2);
      return;
    }
  }

  TilePlan tp[kTilesPerCta];
#pragma unroll
  for (int i = 0; i < kTilesPerCta; ++i) tp[i] = plan_tile<kTilesPerCta>(p, qb, i, sq, skv);
  int nmax = 0;
#pragma unroll
  for (int i = 0; i < kTilesPerCta; ++i) nmax = max(nmax, tp[i].n);

  char* o_head = reinterpret_cast<char*>(p.o) +
                 ((long long)b * p.o_sb + (long long)h * p.o_sh + (long long)q_base * p.o_ss) *
                     (p.out_e4m3 ? 1 : 2);
  float* lse_head =
      p.lse ? p.lse + (long long)b * p.lse_sb + (long long)h * p.lse_sh + q_base : nullptr;

  if (nmax == 0) {
    // Every row of this CTA is fully masked: O = 0, LSE = -inf.
    if (warp < kSoftmaxWarps) {
      const int i = warp / 4;
      const int row = tp[i].q_start + (threadIdx.x % kBlockM);
      if (tp[i].q_start < sq && row < sq) {
        float z[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = 0.f;
        char* row_ptr = o_head + (long long)row * p.o_ss * (p.out_e4m3 ? 1 : 2);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) store_o_chunk(p, row_ptr, c, z);
        if (lse_head) lse_head[row] = -INFINITY;
      }
    }
    return;
  }

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t s_base = ptx::smem_u32(smem);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTilesPerCta; ++i) {
      ptx::mbar_init(&bars.q_full[i], 1);
      ptx::mbar_init(&bars.s_full[i], 1);
      ptx::mbar_init(&bars.s_free[i], 4);
      ptx::mbar_init(&bars.p_full[i], 4);
      ptx::mbar_init(&bars.o_done[i], 1);
    }
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(&bars.kv_full[s], 1);
      ptx::mbar_init(&bars.kv_empty[s], kTilesPerCta);
    }
    for (int i = 0; i < kTilesPerCta; ++i) ptx::mbar_init(&bars.drain[i], 1);
    ptx::mbar_init(&bars.offset, 4);
    abort_sh = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(&tmem_base_sh, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  volatile int* abort_flag = &abort_sh;
  if (threadIdx.x == 0) FA8_TR(2, 63, 1);
  // With FA8_REGS_CONTROL set, registers move from the control warpgroup
  // (TMA / MMA issue) to the two softmax warpgroups; the setmaxnreg sits at
  // the top of each role's branch so the compiler sees one budget per role.
  // 128 x FA8_REGS_CONTROL + 256 x FA8_REGS_SOFTMAX must not exceed the
  // registers the CTA was launched with (Roles<T>::kRegs*).
#if FA8_REGS_CONTROL
#define FA8_REGS_DEC() asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(R::kRegsControl))
#define FA8_REGS_INC() asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(R::kRegsSoftmax))
#else
#define FA8_REGS_DEC() do {} while (0)
#define FA8_REGS_INC() do {} while (0)
#endif

  if (warp >= kSoftmaxWarps) {
  FA8_REGS_DEC();
  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      for (int i = 0; i < kTilesPerCta; ++i) {
        if (tp[i].n == 0) continue;
        ptx::mbar_arrive_expect_tx(&bars.q_full[i], C::kQBytes);
        ptx::tma_load_4d(smem + C::kOffQ + i * C::kQBytes, &tm_q, &bars.q_full[i], 0,
                         q_base + tp[i].q_start, h, tb, pol_q);
      }
      int issued = 0;
      bool ok = true;
      // Loads go in the order the MMA thread consumes them (K0, K1, V0, K2, V1,
      // ..., V(n-1)), so a stage is refilled as soon as the oldest use ends.
      for (int L = 0; L < 2 * nmax && ok && !p.debug_skip_kv_loads; ++L) {
        bool is_v;
        int t;
        load_slot_inverse(L, nmax, is_v, t);
        const int kv = nmax - 1 - t;
        const int st = L % NS;
        if (L >= NS) ok = bounded_wait(&bars.kv_empty[st], ((L / NS) - 1) & 1, abort_flag, p.status, p.timeout_cycles);
        if (!ok) break;
        ptx::mbar_arrive_expect_tx(&bars.kv_full[st], C::kStageBytes);
        uint8_t* dst = smem + C::kOffRing + st * C::kStageBytes;
        if (!is_v)
          ptx::tma_load_4d(dst, &tm_k, &bars.kv_full[st], 0, kv_base + kv * kBlockN, hk, tb,
                           pol_kv);
        else
          ptx::tma_load_4d(dst, &tm_v, &bars.kv_full[st], kv_base + kv * kBlockN, 0, hk, tb,
                           pol_kv);
        ++issued;
      }
      if (!ok) {
        // Drain: wait (bounded) for the last copies issued so that no TMA
        // write lands in shared memory after this CTA exits.
        for (int L = max(0, issued - NS); L < issued; ++L) {
          const long long t0 = clock64();
          while (!ptx::mbar_try_wait(&bars.kv_full[L % NS], (L / NS) & 1) &&
                 clock64() - t0 < p.timeout_cycles) {
          }
        }
        for (int i = 0; i < kTilesPerCta; ++i) {
          if (tp[i].n == 0) continue;
          const long long t0 = clock64();
          while (!ptx::mbar_try_wait(&bars.q_full[i], 0) && clock64() - t0 < p.timeout_cycles) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp || (kTilesPerCta == 2 && warp == kMmaWarp2)) {
    // ------------------------------------------------------------ MMA issuers
    // One issuing thread per query tile (control warp 0: Q0, control warp 2:
    // Q1), so each tile's QK -> softmax -> PV chain advances at its own pace;
    // two softmax warpgroups are not forced into lockstep by a shared in-order
    // issue queue. Every issuer releases every K/V stage (kv_empty counts T).
    if (lane == 0) {
      const int i = (warp == kMmaWarp) ? 0 : 1;
      const uint32_t q_addr = s_base + C::kOffQ + i * C::kQBytes;
      const uint32_t p_hi = s_base + C::kOffP + i * C::kPBytes;
      const uint32_t p_lo = s_base + C::kOffP + (kTilesPerCta + i) * C::kPBytes;
      const int start = nmax - tp[i].n;
      const bool active = tp[i].n > 0;
      const int role = 2 + i;
      bool ok = true;
      if (active) ok = bounded_wait(&bars.q_full[i], 0, abort_flag, p.status, p.timeout_cycles);
      for (int t = -1; t < nmax && ok; ++t) {
        // S_i(t+1) = Q_i K(t+1)^T
        if (i == 0) FA8_TR(2, t + 1, 0);
        if (t + 1 < nmax) {
          const int L = load_slot_k(t + 1);
          const int st = L % NS;
          ok = bounded_wait(&bars.kv_full[st], (L / NS) & 1, abort_flag, p.status, p.timeout_cycles);
          if (!ok) break;
          if (i == 0) FA8_TR(2, t + 1, 1);
          const int tl = t + 1 - start;
          if (active && tl >= 0) {
            if (tl > 0) {
              ok = bounded_wait(&bars.s_free[i], (tl - 1) & 1, abort_flag, p.status, p.timeout_cycles);
              if (!ok) break;
            }
            ptx::tc_fence_after();
            const uint32_t k_addr = s_base + C::kOffRing + st * C::kStageBytes;
            const uint32_t d_tmem = tmem + C::kColS + i * kBlockN;
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk) {
              ptx::umma_f8(d_tmem, ptx::smem_desc_kmajor(q_addr + kk * 32, C::kQKRowBytes),
                           ptx::smem_desc_kmajor(k_addr + kk * 32, C::kQKRowBytes), C::kIdescS,
                           kk > 0 ? 1u : 0u);
            }
            ptx::umma_commit(&bars.s_full[i]);
            if (i == 0) FA8_TR(2, t + 1, 2);
            ptx::umma_commit(&bars.kv_empty[st]);
          } else {
            ptx::mbar_arrive(&bars.kv_empty[st]);
          }
        }
        // O_i += P_i(t) V(t)
        if (t >= 0) {
          const int L = load_slot_v(t, nmax);
          const int st = L % NS;
          ok = bounded_wait(&bars.kv_full[st], (L / NS) & 1, abort_flag, p.status, p.timeout_cycles);
          if (!ok) break;
          if (i == 0) FA8_TR(2, t + 1, 4);
          const int tl = t - start;
          if (active && tl >= 0) {
            ok = bounded_wait(&bars.p_full[i], tl & 1, abort_flag, p.status, p.timeout_cycles);
            if (!ok) break;
            ptx::tc_fence_after();
            const uint32_t v_addr = s_base + C::kOffRing + st * C::kStageBytes;
            const uint32_t d_tmem = tmem + C::kColO + i * D;
            if constexpr (C::kPInTmem) {
              const uint32_t a_hi = tmem + C::kColP;
#pragma unroll
              for (int kk = 0; kk < kBlockN / 32; ++kk)
                ptx::umma_f8_ts(d_tmem, a_hi + kk * 8,
                                ptx::smem_desc_kmajor(v_addr + kk * 32, 128), C::kIdescO,
                                (tl > 0 || kk > 0) ? 1u : 0u);
              if (tp[i].split) {
#pragma unroll
                for (int kk = 0; kk < kBlockN / 32; ++kk)
                  ptx::umma_f8_ts(d_tmem, a_hi + 32 + kk * 8,
                                  ptx::smem_desc_kmajor(v_addr + kk * 32, 128), C::kIdescO, 1u);
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < kBlockN / 32; ++kk) {
                ptx::umma_f8(d_tmem, ptx::smem_desc_kmajor(p_hi + kk * 32, 128),
                             ptx::smem_desc_kmajor(v_addr + kk * 32, 128), C::kIdescO,
                             (tl > 0 || kk > 0) ? 1u : 0u);
              }
              if (tp[i].split) {
#pragma unroll
                for (int kk = 0; kk < kBlockN / 32; ++kk) {
                  ptx::umma_f8(d_tmem, ptx::smem_desc_kmajor(p_lo + kk * 32, 128),
                               ptx::smem_desc_kmajor(v_addr + kk * 32, 128), C::kIdescO, 1u);
                }
              }
            }
            ptx::umma_commit(&bars.o_done[i]);
            if (i == 0) FA8_TR(2, t + 1, 5);
            ptx::umma_commit(&bars.kv_empty[st]);
          } else {
            ptx::mbar_arrive(&bars.kv_empty[st]);
          }
        }
      }
      (void)role;
      // Drain every MMA this thread issued before TMEM is freed.
      ptx::umma_commit(&bars.drain[i]);
      const long long t0 = clock64();
      while (!ptx::mbar_try_wait(&bars.drain[i], 0) && clock64() - t0 < p.timeout_cycles) {
      }
    }
  }
  } else {
    FA8_REGS_INC();
    // ------------------------------------------------------------ softmax WGs
    const int i = warp / 4;                 // query tile of this warpgroup
    const int r = threadIdx.x % kBlockM;    // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + C::kColS + i * kBlockN;
    const uint32_t t_o = tmem + lane_off + C::kColO + i * D;
    const uint32_t p_hi = s_base + C::kOffP + i * C::kPBytes;
    const uint32_t p_lo = s_base + C::kOffP + (kTilesPerCta + i) * C::kPBytes;
    const int n = tp[i].n;
    const int row = tp[i].q_start + r;  // local query row
    const long long row_g = p.q_offset + row;
    float sl2 = p.scale_log2;
    float o_scale = p.o_scale;
    if (p.dq_bh) sl2 *= __ldg(p.dq_bh + b * p.dq_sb + h * p.dq_sh);
    if (p.dk_bh) sl2 *= __ldg(p.dk_bh + b * p.dkv_sb + hk * p.dkv_sh);
    if (p.dv_bh) o_scale *= __ldg(p.dv_bh + b * p.dkv_sb + hk * p.dkv_sh);
    float m_run = -INFINITY;  // running max of s*scale*log2e
    float l_run = 0.f;
    bool ok = true;
    bool offset_sent = false;

    for (int tl = 0; tl < n && ok; ++tl) {
      const int kv = n - 1 - tl;
      if (r == 0) FA8_TR(i, tl, 0);
      ok = bounded_wait(&bars.s_full[i], tl & 1, abort_flag, p.status, p.timeout_cycles);
      if (r == 0) FA8_TR(i, tl, 1);
      if (!ok) break;
      ptx::tc_fence_after();
      float s[kBlockN];
      {
        uint32_t u[kBlockN / 32][32];
#pragma unroll
        for (int c = 0; c < kBlockN / 32; ++c) ptx::tmem_ld32(t_s + c * 32, u[c]);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kBlockN / 32; ++c) {
          ptx::reg_fence32(u[c]);
#pragma unroll
          for (int j = 0; j < 32; ++j) s[c * 32 + j] = __uint_as_float(u[c][j]);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars.s_free[i]);
      if (r == 0) FA8_TR(i, tl, 2);

      // Does any row of this tile need masking at this K/V tile? (keys past
      // seqlen_kv, or, causal, keys after the tile's first query)
      const int kv0 = kv * kBlockN;
      const bool tile_masked =
          (kv0 + kBlockN > skv) ||
          (p.causal && p.kv_offset + kv0 + kBlockN - 1 > p.q_offset + tp[i].q_start);
      uint32_t ph[kBlockN / 4];
      uint32_t pl[kBlockN / 4];
      const bool split = tp[i].split != 0;
      if (kStaggerT && i == 1 && tl == 0) {
        // Start one exp phase behind warpgroup 0 so that one group's barrier
        // waits, S loads and P stores overlap the other's exp work.
        ok = bounded_wait(&bars.offset, 0, abort_flag, p.status, p.timeout_cycles);
        if (!ok) break;
      }
      StepOut so;
      if (!tile_masked && !split) {
        // Hot path: an unmasked K/V tile, single-term P — no mask or split code.
        // D = 128: P conversion fused into the exp loop (+0.6% on C2; D = 64
        // measured 1% slower with it).
        so = softmax_row_step<kBlockN, kEmuPer8, D == 128>(s, sl2, tl == 0, false, m_run, l_run,
                                                           ph, pl);
      } else {
        // Mask: keys past seqlen_kv, and (causal) keys after this query.
        long long lim = skv - kv0;
        if (p.causal) lim = min(lim, row_g - p.kv_offset - kv0 + 1);
        if (lim < kBlockN) {
          const int li = (int)max(lim, -1LL);
#pragma unroll
          for (int c = 0; c < kBlockN; ++c)
            if (c >= li) s[c] = -INFINITY;
        }
        so = softmax_row_step<kBlockN, kEmuPer8>(s, sl2, tl == 0, split, m_run, l_run, ph, pl);
      }
      if (kStaggerT && i == 0 && tl == 0) {
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars.offset);
        offset_sent = true;
      }
#ifdef FA8_TRACE
      if (r == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && tl < 64) {
        fa8_trace_buf[i][tl][6] = so.t_max;  // rescale decision taken
        fa8_trace_buf[i][tl][7] = so.t_exp;  // exponentials and row sum done
      }
#endif
      const bool need = so.need;
      const float alpha = so.alpha;

      // PV(t-1) must be complete before O is rescaled or P overwritten.
      if (r == 0) FA8_TR(i, tl, 3);
      if (tl > 0) {
        ok = bounded_wait(&bars.o_done[i], (tl - 1) & 1, abort_flag, p.status, p.timeout_cycles);
        if (!ok) break;
        if (r == 0) FA8_TR(i, tl, 4);
        if (need) {
          ptx::tc_fence_after();  // TMEM accesses below follow the PV completion
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t u[32];
            ptx::tmem_ld32(t_o + c * 32, u);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(u);
#pragma unroll
            for (int j = 0; j < 32; ++j) u[j] = __float_as_uint(__uint_as_float(u[j]) * alpha);
            ptx::tmem_st32(t_o + c * 32, u);
          }
          ptx::tmem_wait_st();
        }
      }
      if constexpr (C::kPInTmem) {
        // P row -> this lane's 32 TMEM columns (hi) and the next 32 (lo); the
        // stores follow PV(t-1)'s reads of the same columns.
        if (tl > 0 && !need) ptx::tc_fence_after();
        ptx::tmem_st32(tmem + lane_off + C::kColP, ph);
        if (split) ptx::tmem_st32(tmem + lane_off + C::kColP + 32, pl);
        ptx::tmem_wait_st();
      } else {
        const uint32_t row_addr_hi = p_hi + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          ptx::st_shared_v4(row_addr_hi + ((c ^ (r & 7)) << 4), ph[4 * c], ph[4 * c + 1],
                            ph[4 * c + 2], ph[4 * c + 3]);
        if (split) {
          const uint32_t row_addr_lo = p_lo + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            ptx::st_shared_v4(row_addr_lo + ((c ^ (r & 7)) << 4), pl[4 * c], pl[4 * c + 1],
                              pl[4 * c + 2], pl[4 * c + 3]);
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars.p_full[i]);
      if (r == 0) FA8_TR(i, tl, 5);
    }

    if (kStaggerT && i == 0 && !offset_sent) {
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars.offset);
    }
    // Epilogue: O / l -> global, LSE.
    if (r == 0) FA8_TR(i, 63, 0);
    if (n > 0 && ok) ok = bounded_wait(&bars.o_done[i], (n - 1) & 1, abort_flag, p.status, p.timeout_cycles);
    if (r == 0) FA8_TR(i, 63, 1);
    if (tp[i].q_start < sq) {
      ptx::tc_fence_after();
      const float inv_l = (l_run > 0.f && ok) ? o_scale / l_run : 0.f;
      // Whole fp16 tiles go out through the TMA: each thread writes its row
      // into the (now idle) P buffers in the 128B-swizzled box layout, one
      // thread issues the stores. Tiles that end past the sequence (ragged /
      // varlen) and e4m3 output take per-thread global stores.
      const bool tma_out = kTmaStore && p.o_tma && !p.out_e4m3 && n > 0 &&
                           tp[i].q_start + kBlockM <= sq;
      if (tma_out) {
#pragma unroll
        for (int hb = 0; hb < D / 64; ++hb) {
          // box hb = columns [64 hb, 64 hb + 64): 128 rows x 128 B
          const uint32_t box = s_base + C::kOffP + (hb * kTilesPerCta + i) * C::kPBytes;
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t u[32];
            ptx::tmem_ld32(t_o + hb * 64 + c2 * 32, u);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // 4 chunks of 8 halves = 16 B
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __half2 hv = __floats2half2_rn(__uint_as_float(u[8 * j + 2 * e]) * inv_l,
                                               __uint_as_float(u[8 * j + 2 * e + 1]) * inv_l);
                w[e] = *reinterpret_cast<uint32_t*>(&hv);
              }
              const int chunk = c2 * 4 + j;
              ptx::st_shared_v4(box + r * 128 + ((chunk ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
            }
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::named_barrier_sync(1 + i, kBlockM);
        if (r == 0) {
#pragma unroll
          for (int hb = 0; hb < D / 64; ++hb)
            ptx::tma_store_4d(&tm_o, smem + C::kOffP + (hb * kTilesPerCta + i) * C::kPBytes,
                              hb * 64, q_base + tp[i].q_start, h, tb);
          ptx::bulk_commit_group();
          ptx::bulk_wait_group_read0();
        }
      } else {
        char* row_ptr = o_head + (long long)row * p.o_ss * (p.out_e4m3 ? 1 : 2);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          if (n > 0) {
            uint32_t u[32];
            ptx::tmem_ld32(t_o + c * 32, u);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(u);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(u[j]) * inv_l;
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          if (row < sq) store_o_chunk(p, row_ptr, c, v);
        }
      }
      if (lse_head && row < sq) {
        const float base = m_run - kPShift;
        lse_head[row] =
            (l_run > 0.f) ? (__log2f(l_run) + base) * 0.69314718055994531f : -INFINITY;
      }
    }
  }

  if (warp < kSoftmaxWarps && threadIdx.x % kBlockM == 0) FA8_TR(warp / 4, 63, 2);
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FA8_TR(2, 63, 2);
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
#ifdef FA8_TRACE
  if (threadIdx.x == 0 && cta_lin < 4096) fa8_trace_cta[cta_lin][1] = fa8_gtimer();
#endif
}

}  // namespace fa8
