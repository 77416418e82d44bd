// fa8_fwd_kernel.cuh — warp-specialised FP8 (e4m3) flash-attention forward
// for sm_100a.
//
// Replaces the reference's FA2-style Ada kernel flash_attn_fp8_kernel
// (csrc/flash_attention.cu:90-460) and its traits (csrc/kernel_traits.h:11-87)
// with a Blackwell design. A CTA owns one 128-row query tile of one
// (batch, head); two CTAs share an SM (TMEM: 256 columns each, about 97 KB of
// shared memory each), so one CTA's prologue and epilogue overlap the other
// CTA's main loop. 256 threads:
//
//   * warps 0-3 (softmax warpgroup): one thread per query row (= TMEM lane).
//     They run the online softmax in base 2 (the reference's
//     softmax_rescale_o, csrc/flash_attention.cu:54-88, with the scale fixed
//     to softmax_scale * log2(e)), requantise P to e4m3 for the PV product
//     and rescale O in TMEM only when the row max grew by more than
//     kRescaleThreshold (lazy rescale); finally they normalise O by the row
//     sum (the reference's final_softmax_rescale_o,
//     csrc/flash_attention.cu:38-52) and store it;
//   * P is double-buffered (two 128B-swizzled shared tiles for D = 128, two
//     32-column TMEM slots for D = 64, where the PV product reads A from
//     TMEM): P(t) goes to buffer t & 1, so writing it only needs PV(t-2) to
//     be complete, and the e4m3 chunks are stored while the exp loop still
//     runs. PV(t-1) is waited for only when O must be rescaled;
//   * warp 4 (one elected thread) issues tcgen05.mma kind::f8f6f4:
//       S(t+1) = Q K(t+1)^T into TMEM (128 lanes x 128 f32 columns),
//       O += P(t) V(t)     into TMEM (128 lanes x D f32 columns);
//     an MMA issue waits until the tensor pipe accepts it, which is why it
//     has a warp of its own;
//   * warp 5 (TMA producer) streams K and V^T tiles (128 keys each) into a
//     ring of shared stages (cp.async.bulk.tensor, mbarrier completion) in
//     exactly the order the products use them (K0, K1, V0, K2, V1, ...), so
//     every stage is reused first-in first-out. Warps 6-7 only complete the
//     control warpgroup (setmaxnreg works per warpgroup).
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
//     which brings the relative error of P from 2^-4 to about 2^-8. Such
//     tiles use the two P buffers for hi and lo (no double buffering).
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

constexpr int kBlockM = 128;  // query rows per tile (= TMEM lanes)
constexpr int kBlockN = 128;  // keys per K/V tile
constexpr int kThreads = 256;
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kLoadWarp = 5;
constexpr int kMinBlocks = 2;  // CTAs per SM
// setmaxnreg budgets: 128 x kRegsControl + 128 x kRegsSoftmax must not exceed
// the registers the CTA is launched with (65536 / kMinBlocks).
constexpr int kRegsControl = 64;
constexpr int kRegsSoftmax = 192;
static_assert(128 * kRegsControl + 128 * kRegsSoftmax <= 65536 / kMinBlocks,
              "setmaxnreg split exceeds the launch register budget");

#ifndef FA8_EMU128
#define FA8_EMU128 2
#endif
#ifndef FA8_EMU64
#define FA8_EMU64 2
#endif
// Columns of every 8 whose exp2 runs on the FMA pipe instead of MUFU, per head
// dimension (D = 64 has half the tensor work per step for the same number of
// exponentials).
template <int D>
constexpr int kEmuPer8 = (D == 128) ? FA8_EMU128 : FA8_EMU64;
#ifndef FA8_PDBL128
#define FA8_PDBL128 1
#endif
#ifndef FA8_PDBL64
#define FA8_PDBL64 0
#endif
#ifndef FA8_STREAM128
#define FA8_STREAM128 1
#endif
// Double-buffered P (buffer t & 1; writing P(t) waits for PV(t-2)) or one
// buffer (writing P(t) waits for PV(t-1)); streamed e4m3 stores during the exp
// loop for D = 128 (with one buffer they wait for PV(t-1) before the loop).
template <int D>
constexpr bool kPDouble = (D == 128) ? FA8_PDBL128 != 0 : FA8_PDBL64 != 0;
template <int D>
constexpr bool kPStream = D == 128 && FA8_STREAM128 != 0;
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

template <int D>
struct TileCfg {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr int kQKRowBytes = D;              // e4m3 rows of Q and K
  static constexpr int kQBytes = kBlockM * D;
  static constexpr int kStageBytes = kBlockN * D;    // a K tile or a V^T tile (D rows x 128 keys)
  static constexpr int kStages = (D == 128) ? 3 : 8;
  // D = 64 leaves 64 TMEM columns spare: the two P buffers live there (32
  // columns each) and the PV product reads A from TMEM.
  static constexpr bool kPInTmem = FA8_P_TMEM && D == 64;
  static constexpr int kPBytes = kBlockM * kBlockN;  // 128 rows x 128 B (also an O box)
  static constexpr int kPBufs = kPInTmem ? 1 : 2;    // shared P tiles (D = 64: the O box only)
  static constexpr int kOffQ = 0;
  static constexpr int kOffRing = kQBytes;
  static constexpr int kOffP = kOffRing + kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffP + kPBufs * kPBytes;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack for 1024-B alignment
  // TMEM columns: S | O (| P buffer 0 | P buffer 1 for D = 64)
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColO = kBlockN;
  static constexpr uint32_t kTmemCols = 256;
  static constexpr uint32_t kColP = kColO + D;
  static constexpr uint32_t kIdescS = ptx::idesc_e4m3_f32(kBlockM, kBlockN);
  static constexpr uint32_t kIdescO = ptx::idesc_e4m3_f32(kBlockM, D);
  // V stored (B, H_kv, S, D): a V tile is 128 keys x D bytes, exactly like a K
  // tile, and the PV product reads it as an MN-major B operand.
  static constexpr uint32_t kIdescOmn = ptx::idesc_e4m3_f32(kBlockM, D, true);
  static_assert(kPInTmem || D == 128, "D = 64 keeps P in TMEM");
};

struct KernelParams {
  int batch, heads, heads_kv, seqlen_q, seqlen_kv, head_group;
  int causal, out_kind, split_keys, n_qblocks;  // out_kind: 0 fp16, 1 e4m3, 2 fp32
  int o_esize;                                    // bytes per O element
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
  // Split-KV (kv_splits > 1): grid.z = batch * kv_splits; split s of a query
  // tile runs a contiguous share of its K/V tiles and writes a partial
  // (O normalised by its own row sum, fp32, and its LSE) for the tile's last
  // arriving split to merge. Unit u = qtile * kv_splits + s, qtile =
  // (b * heads + h) * n_qblocks + qb.
  int kv_splits;
  float* part_o;             // [units][128][D]
  float* part_lse;           // [units][128]
  unsigned int* split_cnt;   // [qtiles], zero before the launch, left zero after it
};

#ifdef FA8_TRACE
// Debug-only phase timestamps (clock64) of the first kTraceCtas CTAs (linear
// block id): [cta][role][step][event]; roles 0-3 = lane 0 of softmax warps
// 0-3, role 4 = the MMA thread.
constexpr int kTraceCtas = 64;
__device__ long long fa8_trace_buf[kTraceCtas][6][64][8];
// Per-CTA (linear block id < 4096): globaltimer at entry and exit, SM id.
__device__ long long fa8_trace_cta[4096][3];
__device__ __forceinline__ long long fa8_gtimer() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define FA8_TR(role, step, ev)                                                          \
  do {                                                                                  \
    const int cta_tr_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); \
    if (cta_tr_ < kTraceCtas && (step) < 64)                                            \
      fa8_trace_buf[cta_tr_][role][step][ev] = clock64();                               \
  } while (0)
#else
#define FA8_TR(role, step, ev) \
  do {                         \
  } while (0)
#endif

// Barrier slots in static shared memory.
template <int NS>
struct Bars {
  uint64_t q_full;
  uint64_t kv_full[NS];
  uint64_t kv_empty[NS];
  uint64_t s_full;     // S(t) in TMEM (tcgen05.commit of the QK product)
  uint64_t s_free;     // the four softmax warps have read S(t)
  // The four softmax warps have written P(t) (and rescaled O): t even / odd.
  // One barrier per P buffer: a warp may run a step ahead of a slower one
  // (step t+1 only needs PV(t-1) and S(t+1)), and its arrival for P(t+1) must
  // not count toward P(t). It cannot run two steps ahead: step t+2 waits for
  // PV(t), which needs every warp's P(t).
  uint64_t p_full[2];
  uint64_t o_done[2];  // PV(t) complete, t even / odd (the P buffer it read is free)
  uint64_t drain;      // every MMA of the MMA thread has completed
};

// Bounded wait on phase `parity` of `bar`. Returns false on abort/timeout.
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int* status,
                                             long long limit) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
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
// products use them (S(t+1) is issued before O += P(t) V(t)).
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

// Number of K/V tiles the CTA's query tile needs, and whether its P is split.
struct TilePlan {
  int n;        // K/V tiles (tile indices 0 .. n-1)
  int split;    // hi/lo requantisation of P
  int q_start;  // first query row (local)
};

__device__ __forceinline__ TilePlan plan_tile(const KernelParams& p, int qb, int sq, int skv) {
  TilePlan t;
  t.q_start = qb * kBlockM;
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

// Write one row of O (fp16, e4m3 or fp32) from 32 f32 values at column chunk `c`.
__device__ __forceinline__ void store_o_chunk(const KernelParams& p, char* row_ptr, int c,
                                              const float (&v)[32]) {
  if (p.out_kind == 0) {
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
  } else if (p.out_kind == 1) {
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
  } else {
    float4* dst = reinterpret_cast<float4*>(row_ptr + c * 32 * 4);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

constexpr int kMaxKvSplits = 16;

// Store 4 consecutive O values (fp16, e4m3 or fp32) at element offset `col` of a row.
__device__ __forceinline__ void store_o4(const KernelParams& p, char* row_ptr, int col,
                                         float4 v) {
  if (p.out_kind == 0) {
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    *reinterpret_cast<uint2*>(row_ptr + col * 2) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  } else if (p.out_kind == 1) {
    *reinterpret_cast<uint32_t*>(row_ptr + col) =
        (uint32_t)ptx::cvt_e4m3x2(v.x, v.y) | ((uint32_t)ptx::cvt_e4m3x2(v.z, v.w) << 16);
  } else {
    *reinterpret_cast<float4*>(row_ptr + col * 4) = v;
  }
}

// Split-KV tail, run by the 128 softmax threads of every split CTA after each
// wrote its partial row: the last split of the query tile to arrive (atomic
// counter) merges all partials by log-sum-exp,
//   lse = log sum_s exp(lse_s),  O = sum_s exp(lse_s - lse) O_s,
// writes the tile's O and LSE and resets the counter for the next launch.
// The merge first turns each row's LSEs into weights (one thread per row,
// kept in shared memory), then all 128 threads stream the partial rows in
// float4 column groups so that many L2 reads are in flight at once.
template <int D>
__device__ __forceinline__ void split_finish(const KernelParams& p, long long qtile, int r,
                                             int q_start, int sq, char* o_head, float* lse_head,
                                             volatile int* last_sh,
                                             float (*w_sh)[kBlockM]) {
  const int ns = p.kv_splits;
  __threadfence();  // this thread's partial row is visible device-wide
  ptx::named_barrier_sync(3, kBlockM);
  if (r == 0) {
    const unsigned old = atomicAdd(p.split_cnt + qtile, 1u);
    const int last = old == (unsigned)(ns - 1);
    if (last) atomicExch(p.split_cnt + qtile, 0u);
    *last_sh = last;
  }
  ptx::named_barrier_sync(3, kBlockM);
  if (!*last_sh) return;
  __threadfence();
  const long long u0 = qtile * ns;
  {
    float l[kMaxKvSplits];
    float m = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < kMaxKvSplits; ++sp) {
      l[sp] = sp < ns ? __ldcg(p.part_lse + (u0 + sp) * kBlockM + r) : -INFINITY;
      m = fmaxf(m, l[sp]);
    }
    float wsum = 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxKvSplits; ++sp) {
      l[sp] = (m == -INFINITY || l[sp] == -INFINITY) ? 0.f : __expf(l[sp] - m);
      wsum += l[sp];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxKvSplits; ++sp)
      if (sp < ns) w_sh[sp][r] = l[sp] * inv;
    const int row = q_start + r;
    if (lse_head && row < sq) lse_head[row] = wsum > 0.f ? m + __logf(wsum) : -INFINITY;
  }
  ptx::named_barrier_sync(3, kBlockM);
  constexpr int kGroups = D / 4;  // float4 column groups per row
  constexpr int kItems = kBlockM * kGroups / kBlockM;  // column groups per thread
  constexpr int kBatch = 4;  // groups whose loads of every split are in flight together
  static_assert(kItems % kBatch == 0, "batching of the merge");
#pragma unroll 1
  for (int i0 = 0; i0 < kItems; i0 += kBatch) {
    float4 acc[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int s0 = 0; s0 < ns; s0 += 4) {
      float4 x[4][kBatch];
      float w[4][kBatch];
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int i = (i0 + j) * kBlockM + r;
          const int rr = i / kGroups, g = i % kGroups;
          const bool in = s0 + sp < ns;
          w[sp][j] = in ? w_sh[s0 + sp][rr] : 0.f;
          x[sp][j] = in ? __ldcg(reinterpret_cast<const float4*>(
                              p.part_o + ((u0 + s0 + sp) * kBlockM + rr) * D) + g)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          acc[j].x += w[sp][j] * x[sp][j].x;
          acc[j].y += w[sp][j] * x[sp][j].y;
          acc[j].z += w[sp][j] * x[sp][j].z;
          acc[j].w += w[sp][j] * x[sp][j].w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = (i0 + j) * kBlockM + r;
      const int rr = i / kGroups, g = i % kGroups;
      const int row = q_start + rr;
      if (row < sq) store_o4(p, o_head + (long long)row * p.o_ss * p.o_esize, g * 4, acc[j]);
    }
  }
}

// kVmn: V stored (B, H_kv, S, D) and read as an MN-major operand (a
// template parameter so that the MMA issue path carries no layout branch).
template <int D, bool kVmn>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    fa8_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ CUtensorMap tm_o, const KernelParams p) {
  using C = TileCfg<D>;
  constexpr int NS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars<NS> bars;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  __shared__ int softmax_fail_sh;
  __shared__ int split_last_sh;

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
  if (lane == 0 && warp < 6) FA8_TR(warp < 4 ? warp : 4 + (warp == kLoadWarp), 62, 0);
  const int qb = p.causal ? (p.n_qblocks - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z / p.kv_splits;
  const int sidx = blockIdx.z % p.kv_splits;  // split of the K/V range (0 without split-KV)
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
    if ((kv_base & 15) != 0) {
      // A V^T tile must start on a 16-byte boundary (TMA): refuse the sequence.
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, 2);
      return;
    }
    if (sq < 0 || skv < 0 || q_base < 0 || kv_base < 0 || q_base + sq > p.seqlen_q ||
        kv_base + skv > p.seqlen_kv || sq > p.n_qblocks * kBlockM) {
      // Offsets outside the packed tensors, or a sequence longer than
      // max_seqlen_q: refuse the sequence instead of writing out of bounds or
      // leaving rows unwritten silently.
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, 4);
      return;
    }
  }

  const TilePlan tp = plan_tile(p, qb, sq, skv);
  // Split-KV: this CTA runs K/V tiles [t0, t0 + n) of the tile's processing
  // order (tile kv_top - t at local step t).
  int t0 = 0, n = tp.n;
  if (p.kv_splits > 1) {
    t0 = (int)((long long)tp.n * sidx / p.kv_splits);
    n = (int)((long long)tp.n * (sidx + 1) / p.kv_splits) - t0;
  }
  const int kv_top = tp.n - 1 - t0;
  const long long qtile = ((long long)b * p.heads + h) * p.n_qblocks + qb;
  float* const part_o_row0 =
      p.kv_splits > 1 ? p.part_o + (qtile * p.kv_splits + sidx) * kBlockM * D : nullptr;
  float* const part_lse0 =
      p.kv_splits > 1 ? p.part_lse + (qtile * p.kv_splits + sidx) * kBlockM : nullptr;

  char* o_head = reinterpret_cast<char*>(p.o) +
                 ((long long)b * p.o_sb + (long long)h * p.o_sh + (long long)q_base * p.o_ss) *
                     p.o_esize;
  float* lse_head =
      p.lse ? p.lse + (long long)b * p.lse_sb + (long long)h * p.lse_sh + q_base : nullptr;

  // Split-KV merge weights live in the P tiles, idle by the time of the merge.
  float (*const split_w)[kBlockM] = reinterpret_cast<float (*)[kBlockM]>(
      ((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023)) +
      TileCfg<D>::kOffP);
  static_assert(kMaxKvSplits * kBlockM * 4 <= TileCfg<D>::kPBytes, "merge weights fit a P tile");
  if (n == 0 && p.kv_splits > 1) {
    // An empty share of a split query tile: an empty partial, then the merge.
    if (warp < kSoftmaxWarps) {
      const int r = threadIdx.x;
      float4* dst = reinterpret_cast<float4*>(part_o_row0 + (long long)r * D);
#pragma unroll
      for (int j = 0; j < D / 4; ++j) dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      part_lse0[r] = -INFINITY;
      split_finish<D>(p, qtile, r, tp.q_start, sq, o_head, lse_head, &split_last_sh, split_w);
    }
    return;
  }
  if (n == 0) {
    // Every row of this CTA is fully masked (or past the sequence): O = 0, LSE = -inf.
    if (warp < kSoftmaxWarps) {
      const int row = tp.q_start + (int)threadIdx.x;
      if (row < sq) {
        float z[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = 0.f;
        char* row_ptr = o_head + (long long)row * p.o_ss * p.o_esize;
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
  const bool split = tp.split != 0;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars.q_full, 1);
    ptx::mbar_init(&bars.s_full, 1);
    ptx::mbar_init(&bars.s_free, kSoftmaxWarps);
    ptx::mbar_init(&bars.p_full[0], kSoftmaxWarps);
    ptx::mbar_init(&bars.p_full[1], kSoftmaxWarps);
    ptx::mbar_init(&bars.o_done[0], 1);
    ptx::mbar_init(&bars.o_done[1], 1);
    ptx::mbar_init(&bars.drain, 1);
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(&bars.kv_full[s], 1);
      ptx::mbar_init(&bars.kv_empty[s], 1);
    }
    abort_sh = 0;
    softmax_fail_sh = 0;
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
  if (lane == 0 && warp < 6) FA8_TR(warp < 4 ? warp : 4 + (warp == kLoadWarp), 62, 1);

  if (warp >= kSoftmaxWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    if (warp == kLoadWarp && lane == 0) {
      // ---------------------------------------------------------- TMA producer
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(&bars.q_full, C::kQBytes);
      ptx::tma_load_4d(smem + C::kOffQ, &tm_q, &bars.q_full, 0, q_base + tp.q_start, h, tb, pol_q);
      int issued = 0;
      bool ok = true;
      for (int L = 0; L < 2 * n && ok && !p.debug_skip_kv_loads; ++L) {
        bool is_v;
        int t;
        load_slot_inverse(L, n, is_v, t);
        const int kv = kv_top - t;
        const int st = L % NS;
        if (L >= NS)
          ok = bounded_wait(&bars.kv_empty[st], ((L / NS) - 1) & 1, abort_flag, p.status,
                            p.timeout_cycles);
        if (!ok) break;
        ptx::mbar_arrive_expect_tx(&bars.kv_full[st], C::kStageBytes);
        uint8_t* dst = smem + C::kOffRing + st * C::kStageBytes;
        if (!is_v)
          ptx::tma_load_4d(dst, &tm_k, &bars.kv_full[st], 0, kv_base + kv * kBlockN, hk, tb,
                           pol_kv);
        else if (!kVmn)
          ptx::tma_load_4d(dst, &tm_v, &bars.kv_full[st], kv_base + kv * kBlockN, 0, hk, tb,
                           pol_kv);
        else
          ptx::tma_load_4d(dst, &tm_v, &bars.kv_full[st], 0, kv_base + kv * kBlockN, hk, tb,
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
      }
      {
        const long long t0 = clock64();
        while (!ptx::mbar_try_wait(&bars.q_full, 0) && clock64() - t0 < p.timeout_cycles) {
        }
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t q_addr = s_base + C::kOffQ;
      bool ok = bounded_wait(&bars.q_full, 0, abort_flag, p.status, p.timeout_cycles);
      for (int t = -1; t < n && ok; ++t) {
        // S(t+1) = Q K(t+1)^T
        FA8_TR(4, t + 1, 0);
        if (t + 1 < n) {
          const int L = load_slot_k(t + 1);
          const int st = L % NS;
          ok = bounded_wait(&bars.kv_full[st], (L / NS) & 1, abort_flag, p.status, p.timeout_cycles);
          if (!ok) break;
          FA8_TR(4, t + 1, 1);
          if (t + 1 > 0) {
            ok = bounded_wait(&bars.s_free, t & 1, abort_flag, p.status, p.timeout_cycles);
            if (!ok) break;
          }
          ptx::tc_fence_after();
          FA8_TR(4, t + 1, 3);
          const uint32_t k_addr = s_base + C::kOffRing + st * C::kStageBytes;
#pragma unroll
          for (int kk = 0; kk < D / 32; ++kk)
            ptx::umma_f8(tmem + C::kColS, ptx::smem_desc_kmajor(q_addr + kk * 32, C::kQKRowBytes),
                         ptx::smem_desc_kmajor(k_addr + kk * 32, C::kQKRowBytes), C::kIdescS,
                         kk > 0 ? 1u : 0u);
          ptx::umma_commit(&bars.s_full);
          ptx::umma_commit(&bars.kv_empty[st]);
          FA8_TR(4, t + 1, 2);
        }
        // O += P(t) V(t)
        if (t >= 0) {
          const int L = load_slot_v(t, n);
          const int st = L % NS;
          ok = bounded_wait(&bars.kv_full[st], (L / NS) & 1, abort_flag, p.status, p.timeout_cycles);
          if (!ok) break;
          FA8_TR(4, t + 1, 4);
          ok = bounded_wait(&bars.p_full[t & 1], (t >> 1) & 1, abort_flag, p.status, p.timeout_cycles);
          if (!ok) break;
          ptx::tc_fence_after();
          FA8_TR(4, t + 1, 7);
          const uint32_t v_addr = s_base + C::kOffRing + st * C::kStageBytes;
          const uint32_t d_tmem = tmem + C::kColO;
          const int hi_buf = (split || !kPDouble<D>) ? 0 : (t & 1);
          // B = V: K-major V^T tile (D rows of 128 keys) or MN-major V tile
          // (128 rows of D); one K step is 32 keys.
          constexpr uint32_t idesc_o = kVmn ? C::kIdescOmn : C::kIdescO;
          auto desc_v = [&](int kk) -> uint64_t {
            return kVmn ? ptx::smem_desc_mnmajor(v_addr + kk * 32 * D, D)
                            : ptx::smem_desc_kmajor(v_addr + kk * 32, 128);
          };
          if constexpr (C::kPInTmem) {
            const uint32_t a_hi = tmem + C::kColP + 32 * hi_buf;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 32; ++kk)
              ptx::umma_f8_ts(d_tmem, a_hi + kk * 8, desc_v(kk), idesc_o,
                              (t > 0 || kk > 0) ? 1u : 0u);
            if (split) {
#pragma unroll
              for (int kk = 0; kk < kBlockN / 32; ++kk)
                ptx::umma_f8_ts(d_tmem, tmem + C::kColP + 32 + kk * 8, desc_v(kk), idesc_o, 1u);
            }
          } else {
            const uint32_t p_hi = s_base + C::kOffP + hi_buf * C::kPBytes;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 32; ++kk)
              ptx::umma_f8(d_tmem, ptx::smem_desc_kmajor(p_hi + kk * 32, 128), desc_v(kk),
                           idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
            if (split) {
              const uint32_t p_lo = s_base + C::kOffP + C::kPBytes;
#pragma unroll
              for (int kk = 0; kk < kBlockN / 32; ++kk)
                ptx::umma_f8(d_tmem, ptx::smem_desc_kmajor(p_lo + kk * 32, 128), desc_v(kk),
                             idesc_o, 1u);
            }
          }
          ptx::umma_commit(&bars.o_done[t & 1]);
          ptx::umma_commit(&bars.kv_empty[st]);
          FA8_TR(4, t + 1, 5);
        }
      }
      // Drain every MMA this thread issued before TMEM is freed.
      ptx::umma_commit(&bars.drain);
      const long long t0 = clock64();
      while (!ptx::mbar_try_wait(&bars.drain, 0) && clock64() - t0 < p.timeout_cycles) {
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------------ softmax WG
    const int r = threadIdx.x;                          // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t t_s = tmem + lane_off + C::kColS;
    const uint32_t t_o = tmem + lane_off + C::kColO;
    const uint32_t swz = (uint32_t)(r & 7);
    const int row = tp.q_start + r;  // local query row
    const long long row_g = p.q_offset + row;
    float sl2 = p.scale_log2;
    float o_scale = p.o_scale;
    if (p.dq_bh) sl2 *= __ldg(p.dq_bh + b * p.dq_sb + h * p.dq_sh);
    if (p.dk_bh) sl2 *= __ldg(p.dk_bh + b * p.dkv_sb + hk * p.dkv_sh);
    if (p.dv_bh) o_scale *= __ldg(p.dv_bh + b * p.dkv_sb + hk * p.dkv_sh);
    float m_run = -INFINITY;  // running max of s*scale*log2e
    float l_run = 0.f;
    bool ok = true;
    // PV(j) complete: phase j >> 1 of o_done[j & 1].
    auto wait_pv = [&](int j) -> bool {
      return bounded_wait(&bars.o_done[j & 1], (j >> 1) & 1, abort_flag, p.status,
                          p.timeout_cycles);
    };

    for (int tl = 0; tl < n && ok; ++tl) {
      const int kv = kv_top - tl;
      if (lane == 0) FA8_TR(warp, tl, 0);
      ok = bounded_wait(&bars.s_full, tl & 1, abort_flag, p.status, p.timeout_cycles);
      if (lane == 0) FA8_TR(warp, tl, 1);
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
      if (lane == 0) ptx::mbar_arrive(&bars.s_free);
      if (lane == 0) FA8_TR(warp, tl, 2);

      // Does any row of this tile need masking at this K/V tile? (keys past
      // seqlen_kv, or, causal, keys after the tile's first query)
      const int kv0 = kv * kBlockN;
      const bool tile_masked =
          (kv0 + kBlockN > skv) ||
          (p.causal && p.kv_offset + kv0 + kBlockN - 1 > p.q_offset + tp.q_start);
      // P buffer of this step: t & 1 (hi and lo use buffers 0 and 1 when split).
      const bool dbl = kPDouble<D> && !split;
      const int buf = dbl ? (tl & 1) : 0;
      const bool streamed = kPStream<D> && !tile_masked && !split && !C::kPInTmem;
      if (dbl && tl >= 2) {
        // The buffer was read by PV(t-2).
        ok = wait_pv(tl - 2);
        if (!ok) break;
      } else if (!dbl && streamed && tl >= 1) {
        // One buffer, written during the exp loop: PV(t-1) must have read it.
        ok = wait_pv(tl - 1);
        if (!ok) break;
      }
      uint32_t ph[kBlockN / 4];
      uint32_t pl[kBlockN / 4];
      StepOut so;
      if (!tile_masked && !split) {
        // Hot path: an unmasked K/V tile, single-term P — no mask or split
        // code. D = 128: P is converted inside the exp loop and each 16-byte
        // chunk goes to shared memory at once.
        if constexpr (kPStream<D> && !C::kPInTmem)
          so = softmax_row_step<kBlockN, kEmuPer8<D>, true, true>(
              s, sl2, tl == 0, false, m_run, l_run, ph, pl,
              s_base + C::kOffP + buf * C::kPBytes + r * 128, swz);
        else if constexpr (!C::kPInTmem)
          so = softmax_row_step<kBlockN, kEmuPer8<D>, true>(s, sl2, tl == 0, false, m_run, l_run,
                                                           ph, pl);
        else
          so = softmax_row_step<kBlockN, kEmuPer8<D>>(s, sl2, tl == 0, false, m_run, l_run, ph, pl);
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
        so = softmax_row_step<kBlockN, kEmuPer8<D>>(s, sl2, tl == 0, split, m_run, l_run, ph, pl);
      }
#ifdef FA8_TRACE
      {
        const int cta_tr = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        if (lane == 0 && cta_tr < kTraceCtas && tl < 64) {
          fa8_trace_buf[cta_tr][warp][tl][6] = so.t_max;  // rescale decision taken
          fa8_trace_buf[cta_tr][warp][tl][7] = so.t_exp;  // exponentials and row sum done
        }
      }
#endif
      const bool need = so.need;
      const float alpha = so.alpha;

      if (lane == 0) FA8_TR(warp, tl, 3);
      // O may only be rescaled once PV(t-1) is complete; split tiles also
      // reuse PV(t-1)'s buffers.
      if (tl > 0 && (need || !dbl)) {
        ok = wait_pv(tl - 1);
        if (!ok) break;
        if (lane == 0) FA8_TR(warp, tl, 4);
        ptx::tc_fence_after();  // TMEM accesses below follow the PV completion
        if (need) {
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
        // P row -> this lane's 32 TMEM columns of buffer `buf` (hi) and of
        // buffer 1 (lo); the stores follow the reads of the PV product that
        // used them last (waited for above).
        ptx::tc_fence_after();
        ptx::tmem_st32(tmem + lane_off + C::kColP + 32 * buf, ph);
        if (split) ptx::tmem_st32(tmem + lane_off + C::kColP + 32, pl);
        ptx::tmem_wait_st();
      } else {
        if (!streamed) {
          const uint32_t row_addr_hi = s_base + C::kOffP + buf * C::kPBytes + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            ptx::st_shared_v4(row_addr_hi + ((c ^ swz) << 4), ph[4 * c], ph[4 * c + 1],
                              ph[4 * c + 2], ph[4 * c + 3]);
          if (split) {
            const uint32_t row_addr_lo = s_base + C::kOffP + C::kPBytes + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
              ptx::st_shared_v4(row_addr_lo + ((c ^ swz) << 4), pl[4 * c], pl[4 * c + 1],
                                pl[4 * c + 2], pl[4 * c + 3]);
          }
        }
        ptx::fence_proxy_async_smem();
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars.p_full[tl & 1]);
      if (lane == 0) FA8_TR(warp, tl, 5);
    }
    ok = __all_sync(0xffffffffu, ok);

    // Epilogue: O / l -> global, LSE.
    if (lane == 0) FA8_TR(warp, 62, 2);
    if (ok) ok = wait_pv(n - 1);
    if (lane == 0) FA8_TR(warp, 62, 3);
    ok = __all_sync(0xffffffffu, ok);
    // One CTA-wide verdict for the four softmax warps (the TMA-store path
    // below has a barrier that all of them must reach).
    if (!ok && lane == 0) softmax_fail_sh = 1;
    ptx::named_barrier_sync(1, kBlockM);
    ok = ok && (*static_cast<volatile int*>(&softmax_fail_sh) == 0);
    ptx::tc_fence_after();
    const float inv_l = (l_run > 0.f && ok) ? o_scale / l_run : 0.f;
    // Whole fp16 tiles go out through the TMA: each thread writes its row into
    // the P tiles (idle once the last PV completed) in the 128B-swizzled box
    // layout, one thread issues the stores. Tiles that end past the sequence (ragged /
    // varlen), e4m3 output and aborted CTAs take per-thread global stores.
    const bool tma_out = kTmaStore && p.o_tma && p.out_kind == 0 && ok &&
                         tp.q_start + kBlockM <= sq && p.kv_splits == 1;
    if (p.kv_splits > 1) {
      // Partial of this split: O / l (fp32) and its LSE; the merge follows below.
      float4* dst = reinterpret_cast<float4*>(part_o_row0 + (long long)r * D);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        ptx::tmem_ld32(t_o + c * 32, u);
        ptx::tmem_wait_ld();
        ptx::reg_fence32(u);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[c * 8 + j] = ok ? make_float4(__uint_as_float(u[4 * j]) * inv_l,
                                            __uint_as_float(u[4 * j + 1]) * inv_l,
                                            __uint_as_float(u[4 * j + 2]) * inv_l,
                                            __uint_as_float(u[4 * j + 3]) * inv_l)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const float base = m_run - kPShift;
      part_lse0[r] =
          (l_run > 0.f && ok) ? (__log2f(l_run) + base) * 0.69314718055994531f : -INFINITY;
      split_finish<D>(p, qtile, r, tp.q_start, sq, o_head, lse_head, &split_last_sh, split_w);
    } else if (tma_out) {
#pragma unroll
      for (int hb = 0; hb < D / 64; ++hb) {
        // box hb = columns [64 hb, 64 hb + 64): 128 rows x 128 B
        const uint32_t box = s_base + C::kOffP + hb * C::kPBytes;
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
      ptx::named_barrier_sync(2, kBlockM);
      if (r == 0) {
#pragma unroll
        for (int hb = 0; hb < D / 64; ++hb)
          ptx::tma_store_4d(&tm_o, smem + C::kOffP + hb * C::kPBytes, hb * 64,
                            q_base + tp.q_start, h, tb);
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_read0();
      }
    } else {
      char* row_ptr = o_head + (long long)row * p.o_ss * p.o_esize;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        uint32_t u[32];
        ptx::tmem_ld32(t_o + c * 32, u);
        ptx::tmem_wait_ld();
        ptx::reg_fence32(u);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = ok ? __uint_as_float(u[j]) * inv_l : 0.f;
        if (row < sq) store_o_chunk(p, row_ptr, c, v);
      }
    }
    if (lse_head && row < sq && p.kv_splits == 1) {
      const float base = m_run - kPShift;
      lse_head[row] =
          (l_run > 0.f && ok) ? (__log2f(l_run) + base) * 0.69314718055994531f : -INFINITY;
    }
  }

  if (lane == 0 && warp < 6) FA8_TR(warp < 4 ? warp : 4 + (warp == kLoadWarp), 62, 4);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
  if (lane == 0 && warp < 6) FA8_TR(warp < 4 ? warp : 4 + (warp == kLoadWarp), 62, 5);
#ifdef FA8_TRACE
  if (threadIdx.x == 0 && cta_lin < 4096) fa8_trace_cta[cta_lin][1] = fa8_gtimer();
#endif
}

}  // namespace fa8
