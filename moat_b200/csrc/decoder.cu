// Decoder-step glue for the INT4 decode path on B200 (sm_100a): the element-wise and
// row-wise operations between the INT4 GEMMs and the LUT attention of one decode step.
//
// Reference semantics (antigravity-engine/src/transformer.py):
//   RMSNorm            :26-37   x * rsqrt(mean(x^2) + eps) * weight (fp32 math)
//   RoPE               :39-63   adjacent pairs (x[2i], x[2i+1]) rotated by pos * theta^(-2i/d)
//   SwiGLU MLP         :124-134 down(silu(gate(x)) * up(x))
//   residual adds, embedding lookup, greedy argmax (batch_generator.py:203-206, 224-227).
// The residual stream is kept in fp32; every GEMM input is rounded to fp16 once.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"

namespace mb {

constexpr int kRowBlock = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x[n, :] = float(table[ids[n], :])
__global__ void __launch_bounds__(kRowBlock) k_embed(const int32_t* __restrict__ ids, const uint16_t* __restrict__ table,
                                                     int D, int V, float* __restrict__ x, uint32_t* err) {
  pdl_wait();  // the ids may come from the previous step's argmax
  pdl_launch_dependents();
  const int n = blockIdx.x;
  const int id = ids[n];
  if (id < 0 || id >= V) {  // out-of-range token: zero row, error bit
    if (threadIdx.x == 0 && err) atomicOr(err, MB_DEVERR_INDEX);
    for (int c = threadIdx.x; c < D; c += kRowBlock) x[static_cast<int64_t>(n) * D + c] = 0.0f;
    return;
  }
  const uint16_t* row = table + static_cast<int64_t>(id) * D;
  for (int c = threadIdx.x; c < D; c += kRowBlock)
    x[static_cast<int64_t>(n) * D + c] = __half2float(__ushort_as_half(row[c]));
}

// x += y (if y), then h = fp16(x * rsqrt(mean(x^2) + eps) * w); one CTA per row.
__global__ void __launch_bounds__(kRowBlock) k_add_rmsnorm(float* __restrict__ x, const uint16_t* __restrict__ y,
                                                           const float* __restrict__ w, int D, float eps,
                                                           uint16_t* __restrict__ h) {
  __shared__ float part[kRowBlock / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  float* xr = x + static_cast<int64_t>(n) * D;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < D; c += kRowBlock) {
    float v = xr[c];
    if (y) {
      v += __half2float(__ushort_as_half(y[static_cast<int64_t>(n) * D + c]));
      xr[c] = v;
    }
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kRowBlock / 32; ++i) tot += part[i];  // fixed order: deterministic
  const float inv = rsqrtf(tot / static_cast<float>(D) + eps);
  for (int c = threadIdx.x; c < D; c += kRowBlock)
    h[static_cast<int64_t>(n) * D + c] = __half_as_ushort(__float2half_rn(xr[c] * inv * w[c]));
}

// qkv [N, 3*H*dh] fp16 (q | k | v, heads contiguous). For trace n, head hh at
// position pos[n]: q_out[n, hh] = rope(q), k_cache[n, hh, pos] = rope(k),
// v_cache[n, hh, pos] = v. Pair i = (x[2i], x[2i+1]) rotates by angle pos * f_i with
// (cos, sin) read from cs[pos][i] (fp32, built on the host). One CTA per (n, head).
__global__ void __launch_bounds__(64) k_rope_append(const uint16_t* __restrict__ qkv, int H, int dh,
                                                    const int32_t* __restrict__ pos, const float2* __restrict__ cs,
                                                    int Lmax, uint16_t* __restrict__ q_out, uint16_t* __restrict__ kc,
                                                    uint16_t* __restrict__ vc, uint32_t* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x / H, hh = blockIdx.x % H;
  const int p = pos[n];
  const int HD = H * dh;
  const uint16_t* base = qkv + static_cast<int64_t>(n) * 3 * HD + hh * dh;
  if (p < 0 || p >= Lmax) {
    if (threadIdx.x == 0 && err) atomicOr(err, MB_DEVERR_INDEX);
    return;
  }
  const int64_t crow = (static_cast<int64_t>(n) * H + hh) * Lmax + p;  // cache row of this position
  for (int i = threadIdx.x; i < dh / 2; i += blockDim.x) {
    const float2 r = cs[static_cast<int64_t>(p) * (dh / 2) + i];
    const __half2 q2 = *reinterpret_cast<const __half2*>(base + 2 * i);
    const __half2 k2 = *reinterpret_cast<const __half2*>(base + HD + 2 * i);
    const float2 qf = __half22float2(q2), kf = __half22float2(k2);
    const float2 qo = make_float2(qf.x * r.x - qf.y * r.y, qf.x * r.y + qf.y * r.x);
    const float2 ko = make_float2(kf.x * r.x - kf.y * r.y, kf.x * r.y + kf.y * r.x);
    *reinterpret_cast<__half2*>(q_out + (static_cast<int64_t>(n) * H + hh) * dh + 2 * i) = __floats2half2_rn(qo.x, qo.y);
    *reinterpret_cast<__half2*>(kc + crow * dh + 2 * i) = __floats2half2_rn(ko.x, ko.y);
    *reinterpret_cast<uint32_t*>(vc + crow * dh + 2 * i) = *reinterpret_cast<const uint32_t*>(base + 2 * HD + 2 * i);
  }
}

// a[n, j] = fp16(silu(g) * u) with g = gu[n, j], u = gu[n, F + j] (fp32 math).
__global__ void __launch_bounds__(kRowBlock) k_swiglu(const uint16_t* __restrict__ gu, int F, int64_t total,
                                                      uint16_t* __restrict__ a) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t e = blockIdx.x * static_cast<int64_t>(kRowBlock) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * kRowBlock) {
    const int64_t n = e / F;
    const int j = static_cast<int>(e - n * F);
    const float g = __half2float(__ushort_as_half(gu[n * 2 * F + j]));
    const float u = __half2float(__ushort_as_half(gu[n * 2 * F + F + j]));
    const float s = g / (1.0f + expf(-g));
    a[e] = __half_as_ushort(__float2half_rn(s * u));
  }
}

// ids[n] = first index of the largest logit of row n (a NaN counts as the largest,
// -0 equals +0, like numpy.argmax). One CTA of 1024 threads per row.
constexpr int kArgBlock = 1024;

__device__ __forceinline__ unsigned long long block_best_key(unsigned long long best, unsigned long long* best_w) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) best_w[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < kArgBlock / 32; ++w) best = best_w[w] > best ? best_w[w] : best;
  return best;  // the row's best key in thread 0
}

__global__ void __launch_bounds__(kArgBlock) k_argmax(const uint16_t* __restrict__ logits, int V,
                                                      int32_t* __restrict__ ids) {
  __shared__ unsigned long long best_w[kArgBlock / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  const unsigned long long best =
      block_best_key(thread_best_key(logits + static_cast<int64_t>(n) * V, V, 0, threadIdx.x, kArgBlock), best_w);
  if (threadIdx.x == 0) ids[n] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
}

// One row shard of a column-split vocabulary: the shard's best logit as a 64-bit key,
// code << 32 | (0xFFFFFFFF - global column). The largest key over all shards is the
// global argmax with ties to the first column, so the shards combine with one integer
// MAX all-reduce.
__global__ void __launch_bounds__(kArgBlock) k_argmax_key(const uint16_t* __restrict__ logits, int V, int col0,
                                                          int64_t* __restrict__ keys) {
  __shared__ unsigned long long best_w[kArgBlock / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  const unsigned long long best =
      block_best_key(thread_best_key(logits + static_cast<int64_t>(n) * V, V, col0, threadIdx.x, kArgBlock), best_w);
  if (threadIdx.x == 0) keys[n] = static_cast<int64_t>(best);
}

__global__ void k_keys_to_ids(const int64_t* __restrict__ keys, int N, int32_t* __restrict__ ids) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n < N) ids[n] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(keys[n] & 0xFFFFFFFFll));
}

// pos[n] += 1 (the next step's position), on the device so a captured step can replay.
__global__ void k_advance(int32_t* pos, int N) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n < N) pos[n] += 1;
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_embed(const int32_t* ids, int32_t N, const uint16_t* table, int32_t V, int32_t D, float* x,
                 uint32_t* dev_err, void* stream) {
  if (!ids || !table || !x) return MB_ERR_NULL;
  if (N < 1 || V < 1 || D < 1) return MB_ERR_ARGS;
  return launch_with_pdl(k_embed, dim3(N), dim3(kRowBlock), 0, static_cast<cudaStream_t>(stream), ids, table, D, V, x,
                         dev_err);
}

int32_t mb_add_rmsnorm(float* x, const uint16_t* y, const float* w, int32_t N, int32_t D, float eps, uint16_t* h,
                       void* stream) {
  if (!x || !w || !h) return MB_ERR_NULL;
  if (N < 1 || D < 1 || !(eps >= 0.0f)) return MB_ERR_ARGS;
  return launch_with_pdl(k_add_rmsnorm, dim3(N), dim3(kRowBlock), 0, static_cast<cudaStream_t>(stream), x, y, w, D,
                         eps, h);
}

int32_t mb_rope_append(const uint16_t* qkv, int32_t N, int32_t H, int32_t dh, const int32_t* pos, const float* cs,
                       int32_t Lmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, uint32_t* dev_err,
                       void* stream) {
  if (!qkv || !pos || !cs || !q_out || !k_cache || !v_cache) return MB_ERR_NULL;
  if (N < 1 || H < 1 || dh < 2 || dh % 2 != 0 || Lmax < 1) return MB_ERR_ARGS;
  if (!aligned(qkv, 4) || !aligned(q_out, 4) || !aligned(k_cache, 4) || !aligned(v_cache, 4) || !aligned(cs, 8))
    return MB_ERR_ALIGN;
  return launch_with_pdl(k_rope_append, dim3(N * H), dim3(64), 0, static_cast<cudaStream_t>(stream), qkv, H, dh, pos,
                         reinterpret_cast<const float2*>(cs), Lmax, q_out, k_cache, v_cache, dev_err);
}

int32_t mb_swiglu(const uint16_t* gu, int32_t N, int32_t F, uint16_t* a, void* stream) {
  if (!gu || !a) return MB_ERR_NULL;
  if (N < 1 || F < 1) return MB_ERR_ARGS;
  const int64_t total = static_cast<int64_t>(N) * F;
  const int64_t blocks = std::min<int64_t>((total + kRowBlock - 1) / kRowBlock, static_cast<int64_t>(sm_count()) * 8);
  return launch_with_pdl(k_swiglu, dim3(static_cast<unsigned>(blocks)), dim3(kRowBlock), 0,
                         static_cast<cudaStream_t>(stream), gu, F, total, a);
}

int32_t mb_argmax_f16(const uint16_t* logits, int32_t N, int32_t V, int32_t* ids, void* stream) {
  if (!logits || !ids) return MB_ERR_NULL;
  if (N < 1 || V < 1) return MB_ERR_ARGS;
  return launch_with_pdl(k_argmax, dim3(N), dim3(kArgBlock), 0, static_cast<cudaStream_t>(stream), logits, V, ids);
}

int32_t mb_argmax_key_f16(const uint16_t* logits, int32_t N, int32_t V, int32_t col0, int64_t* keys, void* stream) {
  if (!logits || !keys) return MB_ERR_NULL;
  if (N < 1 || V < 1 || col0 < 0 || static_cast<int64_t>(col0) + V > 0x7FFFFFFFll) return MB_ERR_ARGS;
  return launch_with_pdl(k_argmax_key, dim3(N), dim3(kArgBlock), 0, static_cast<cudaStream_t>(stream), logits, V,
                         col0, keys);
}

int32_t mb_argmax_keys_to_ids(const int64_t* keys, int32_t N, int32_t* ids, void* stream) {
  if (!keys || !ids) return MB_ERR_NULL;
  if (N < 1) return MB_ERR_ARGS;
  return launch_with_pdl(k_keys_to_ids, dim3((N + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream), keys,
                         N, ids);
}

int32_t mb_advance_positions(int32_t* pos, int32_t N, void* stream) {
  if (!pos) return MB_ERR_NULL;
  if (N < 1) return MB_ERR_ARGS;
  return launch_with_pdl(k_advance, dim3((N + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream), pos, N);
}

}  // extern "C"
