// fa8_aux.cu — the two kernels either side of the attention forward:
//
//  * fa8_lse_merge: combines partial (O_i, LSE_i) of the same query rows —
//    the exchange step of the context-parallel ring. Each partial is an
//    attention output normalised over its own key block, so
//        lse = log sum_i exp(lse_i),   o = sum_i exp(lse_i - lse) o_i.
//    The reference has no counterpart (it emits no LSE).
//  * fa8_quantize_e4m3: fp16/bf16 -> e4m3 (RNE, saturating), optionally
//    transposing each (rows x cols) matrix — the casts and V transpose the
//    reference's test.py performs with torch (test.py:35-37, :51-52).
//
// Both are HBM-bound elementwise passes: 16-byte vector accesses, one
// thread per 8 (merge) or 16 (quantise) output elements, grids sized in
// multiples of the SM count via grid-stride loops; the transposing quantise
// moves 64 x 64 tiles through shared memory with 16-byte global accesses.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/fa8.h"
#include "sm100_ptx.cuh"

void fa8_note_launch();
int fa8_note_cuda_error(cudaError_t e, const char* where);
int fa8_note_error(int status, const char* msg);

namespace {

constexpr int kMaxParts = 16;

struct MergeArgs {
  const void* o[kMaxParts];
  const float* lse[kMaxParts];
};

// One thread = 8 consecutive elements of one row.
__global__ void lse_merge_kernel(MergeArgs a, int n, int o_f16, int64_t rows, int hd,
                                 __half* out, int64_t out_stride, float* lse_out) {
  const int per_row = hd / 8;
  const int64_t total = rows * per_row;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / per_row;
    const int c0 = (int)(idx % per_row) * 8;
    float m = -INFINITY;
    for (int i = 0; i < n; ++i) m = fmaxf(m, a.lse[i][row]);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    if (m != -INFINITY) {
      for (int i = 0; i < n; ++i) {
        const float l = a.lse[i][row];
        if (l == -INFINITY) continue;
        const float w = __expf(l - m);
        wsum += w;
        if (o_f16) {
          const uint4 raw =
              *reinterpret_cast<const uint4*>(static_cast<const __half*>(a.o[i]) + row * hd + c0);
          const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
            acc[2 * e] += w * f.x;
            acc[2 * e + 1] += w * f.y;
          }
        } else {
          const float4* src =
              reinterpret_cast<const float4*>(static_cast<const float*>(a.o[i]) + row * hd + c0);
          const float4 x0 = src[0], x1 = src[1];
          acc[0] += w * x0.x; acc[1] += w * x0.y; acc[2] += w * x0.z; acc[3] += w * x0.w;
          acc[4] += w * x1.x; acc[5] += w * x1.y; acc[6] += w * x1.z; acc[7] += w * x1.w;
        }
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    uint32_t w4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __half2 hv = __floats2half2_rn(acc[2 * e] * inv, acc[2 * e + 1] * inv);
      w4[e] = *reinterpret_cast<uint32_t*>(&hv);
    }
    *reinterpret_cast<uint4*>(out + row * out_stride + c0) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    if (lse_out && c0 == 0) lse_out[row] = (wsum > 0.f) ? m + __logf(wsum) : -INFINITY;
  }
}

__device__ __forceinline__ float load_in(const void* x, int dt, int64_t i) {
  return dt == 0 ? __half2float(static_cast<const __half*>(x)[i])
                 : (dt == 1 ? __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i])
                            : 0.f);
}

// Row-major quantise: one thread = 16 consecutive elements (cols % 16 == 0).
__global__ void quantize_kernel(const void* x, int dt, uint8_t* y, int64_t n16, float scale) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n16;
       idx += (int64_t)gridDim.x * blockDim.x) {
    float v[16];
    if (dt == 0) {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + idx * 16);
      const uint4 r0 = src[0], r1 = src[1];
      const __half2* h0 = reinterpret_cast<const __half2*>(&r0);
      const __half2* h1 = reinterpret_cast<const __half2*>(&r1);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __half22float2(h0[e]);
        v[2 * e] = f.x; v[2 * e + 1] = f.y;
        f = __half22float2(h1[e]);
        v[8 + 2 * e] = f.x; v[8 + 2 * e + 1] = f.y;
      }
    } else {
      const uint4* src =
          reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + idx * 16);
      const uint4 r0 = src[0], r1 = src[1];
      const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&r0);
      const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&r1);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h0[e]);
        v[2 * e] = f.x; v[2 * e + 1] = f.y;
        f = __bfloat1622float2(h1[e]);
        v[8 + 2 * e] = f.x; v[8 + 2 * e + 1] = f.y;
      }
    }
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = (uint32_t)fa8::ptx::cvt_e4m3x2(v[4 * e] * scale, v[4 * e + 1] * scale) |
             ((uint32_t)fa8::ptx::cvt_e4m3x2(v[4 * e + 2] * scale, v[4 * e + 3] * scale) << 16);
    reinterpret_cast<uint4*>(y)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Transposing quantise of whole 64 x 64 tiles with 16-byte global accesses on
// both sides: x[b][r][c] (fp16/bf16, cols % 8 == 0) -> y[b][c][r] (e4m3, rows
// % 16 == 0). Each thread loads 8 consecutive input elements of one row (16 B),
// quantises them and scatters the 8 bytes into a transposed shared tile; after
// the barrier each thread writes 16 consecutive output bytes of one output row.
__global__ void quantize_transpose_vec_kernel(const void* x, int dt, uint8_t* y, int64_t rows,
                                              int64_t cols, float scale) {
  constexpr int kPad = 16;  // row pitch 80 B: keeps the 16-byte reads aligned
  __shared__ __align__(16) uint8_t tile_t[64][64 + kPad];  // [c][r]
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int64_t base = b * rows * cols;
  // 64 rows x 8 vectors of 8 elements = 512 vectors, two per thread.
  for (int e = threadIdx.x; e < 512; e += blockDim.x) {
    const int rr = e / 8, cv = (e % 8) * 8;
    const int64_t r = r0 + rr, c = c0 + cv;
    float v[8];
    if (r < rows && c < cols) {  // cols % 8 == 0: the vector is all in or all out
      const uint4 raw = *reinterpret_cast<const uint4*>(
          static_cast<const char*>(x) + (base + r * cols + c) * 2);
      if (dt == 0) {
        const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(h[k]);
          v[2 * k] = f.x;
          v[2 * k + 1] = f.y;
        }
      } else {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          v[2 * k] = f.x;
          v[2 * k + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      const uint16_t two = fa8::ptx::cvt_e4m3x2(v[k] * scale, v[k + 1] * scale);
      tile_t[cv + k][rr] = (uint8_t)(two & 0xffu);
      tile_t[cv + k + 1][rr] = (uint8_t)(two >> 8);
    }
  }
  __syncthreads();
  // 64 output rows x 4 vectors of 16 bytes = 256 vectors, one per thread.
  for (int e = threadIdx.x; e < 256; e += blockDim.x) {
    const int cc = e / 4, rv = (e % 4) * 16;
    const int64_t c = c0 + cc, r = r0 + rv;
    if (c < cols && r < rows)  // rows % 16 == 0: the vector is all in or all out
      *reinterpret_cast<uint4*>(y + base + c * rows + r) =
          *reinterpret_cast<const uint4*>(&tile_t[cc][rv]);
  }
}

// Transposing quantise through a 64x64 shared tile, one element per access:
// the fallback for shapes or pointers the vector kernel cannot take.
__global__ void quantize_transpose_kernel(const void* x, int dt, uint8_t* y, int64_t rows,
                                          int64_t cols, float scale) {
  __shared__ uint8_t tile[64][64 + 4];
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int64_t base = b * rows * cols;
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int rr = e / 64, cc = e % 64;
    const int64_t r = r0 + rr, c = c0 + cc;
    uint8_t q = 0;
    if (r < rows && c < cols) {
      const float f = load_in(x, dt, base + r * cols + c) * scale;
      q = (uint8_t)(fa8::ptx::cvt_e4m3x2(f, 0.f) & 0xffu);
    }
    tile[rr][cc] = q;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int cc = e / 64, rr = e % 64;
    const int64_t r = r0 + rr, c = c0 + cc;
    if (r < rows && c < cols) y[base + c * rows + r] = tile[rr][cc];
  }
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace

extern "C" int fa8_lse_merge(int n_parts, const void* const* o_parts, int o_is_f16,
                             const float* const* lse_parts, int64_t rows, int64_t head_dim,
                             void* o_out, int64_t o_out_stride, float* lse_out, void* stream) {
  if (n_parts < 1 || n_parts > kMaxParts || !o_parts || !lse_parts || !o_out)
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_lse_merge: bad part list");
  if (rows < 0 || head_dim <= 0 || head_dim % 8 != 0 || o_out_stride < head_dim ||
      o_out_stride % 8 != 0)
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_lse_merge: bad shape");
  if (rows == 0) return FA8_OK;
  MergeArgs a;
  for (int i = 0; i < kMaxParts; ++i) {
    a.o[i] = i < n_parts ? o_parts[i] : nullptr;
    a.lse[i] = i < n_parts ? lse_parts[i] : nullptr;
    if (i < n_parts && (!a.o[i] || !a.lse[i]))
      return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_lse_merge: null part");
    // Parts are read and O is written with 16-byte vector accesses.
    if (i < n_parts && (reinterpret_cast<uintptr_t>(a.o[i]) & 15))
      return fa8_note_error(FA8_ERR_ALIGNMENT, "fa8_lse_merge: o_parts must be 16-byte aligned");
  }
  if (reinterpret_cast<uintptr_t>(o_out) & 15)
    return fa8_note_error(FA8_ERR_ALIGNMENT, "fa8_lse_merge: o_out must be 16-byte aligned");
  const int64_t total = rows * (head_dim / 8);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  lse_merge_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      a, n_parts, o_is_f16, rows, (int)head_dim, static_cast<__half*>(o_out), o_out_stride,
      lse_out);
  fa8_note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA8_OK : fa8_note_cuda_error(e, "lse_merge_kernel launch");
}

extern "C" int fa8_quantize_e4m3(const void* x, int in_dtype, void* y, int64_t batch,
                                 int64_t rows, int64_t cols, float scale, int transpose,
                                 void* stream) {
  if (!x || !y || batch < 0 || rows < 0 || cols < 0 || (in_dtype != 0 && in_dtype != 1))
    return fa8_note_error(FA8_ERR_INVALID_ARG, "fa8_quantize_e4m3: bad arguments");
  if (batch == 0 || rows == 0 || cols == 0) return FA8_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!transpose) {
    const int64_t n = batch * rows * cols;
    if (n % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
      return fa8_note_error(FA8_ERR_ALIGNMENT,
                            "fa8_quantize_e4m3: element count must be a multiple of 16 and "
                            "buffers 16-byte aligned");
    const int threads = 256;
    int64_t blocks = (n / 16 + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    quantize_kernel<<<(unsigned)blocks, threads, 0, s>>>(x, in_dtype, static_cast<uint8_t*>(y),
                                                         n / 16, scale);
  } else {
    if (batch > 65535 || (rows + 63) / 64 > 65535)
      return fa8_note_error(FA8_ERR_UNSUPPORTED, "fa8_quantize_e4m3: transpose grid too large");
    dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64), (unsigned)batch);
    const bool vec = rows % 16 == 0 && cols % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    if (vec)
      quantize_transpose_vec_kernel<<<grid, 256, 0, s>>>(x, in_dtype, static_cast<uint8_t*>(y),
                                                         rows, cols, scale);
    else
      quantize_transpose_kernel<<<grid, 256, 0, s>>>(x, in_dtype, static_cast<uint8_t*>(y),
                                                     rows, cols, scale);
  }
  fa8_note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA8_OK : fa8_note_cuda_error(e, "quantize kernel launch");
}
