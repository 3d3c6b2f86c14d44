// Exp-LUT softmax and split-KV decode attention for B200 (sm_100a).
//
// Reference semantics: ExponentialLUT.lookup / safe_softmax_lut
// (antigravity-engine/src/attention.py:60-85, 97-134) and the decode attention the
// reference composes from gqa_attention_scores_kernel (transformer_ops.metal:94-123),
// the LUT softmax, and attention_value_kernel (transformer_ops.metal:186-214).
//
// The LUT index must match the reference bit for bit, so the exponent is never
// recomputed on the device: idx = trunc(min(|x| / step, size - 1)) with an IEEE
// fp32 divide (__fdiv_rn) by step = fp32(range_max / (size - 1)), and the value is
// table[size - 1 - idx]. Because the LUT argument is x - max over the WHOLE row,
// the attention runs in three streaming passes instead of an online softmax:
//   1. scores  (streams K): s_l = (q . k_l) * scale -> fp32 workspace, chunk maxima
//   2. stats   (reads the 4 MB of scores from L2): row max, sum of LUT values
//   3. p . V   (streams V): p_l = fp16(LUT(s_l - max) / sum), fp32 sum of p_l v_l per
//      chunk into a per-chunk slot; the last chunk to arrive sums the slots in chunk
//      order (deterministic) and writes the fp16 output. The workspace needs no
//      initial contents (pass 1 resets the arrival counters).
// Rows of up to 2048 keys (the decode step's caches) take one launch instead: one CTA
// per row streams its K and then its V rows through a shared-memory ring with bulk
// copies, holding the row's scores in shared memory (k_attn_stream); with fewer rows
// than SMs, a cluster of CTAs shares each row (k_attn_stream_split).
#include <algorithm>

#include "common.cuh"

namespace mb {

__device__ __forceinline__ int lut_index(float x, float step, int size) {
  float f = __fdiv_rn(fabsf(x), step);
  f = fminf(fmaxf(f, 0.0f), static_cast<float>(size - 1));
  return static_cast<int>(f);  // truncation toward zero
}

__device__ __forceinline__ float lut_exp(const uint16_t* __restrict__ table, float x, float step, int size) {
  return __half2float(__ushort_as_half(__ldg(table + (size - 1 - lut_index(x, step, size)))));
}

__device__ __forceinline__ float nanmax_f(float a, float b) { return (b > a || b != b) ? b : a; }

template <int BLOCK>
__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = nanmax_f(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < BLOCK / 32) ? sh[threadIdx.x] : -INFINITY;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = nanmax_f(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

template <int BLOCK>
__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < BLOCK / 32) ? sh[threadIdx.x] : 0.0f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

__global__ void __launch_bounds__(256) k_lut_lookup(const uint16_t* __restrict__ table, int size, float step,
                                                    const float* __restrict__ x, int64_t n, uint16_t* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __ldg(table + (size - 1 - lut_index(x[i], step, size)));
}

// One CTA per row: max, LUT exp + fp32 sum, normalise to fp16.
__global__ void __launch_bounds__(256) k_lut_softmax(const float* __restrict__ x, int64_t cols,
                                                     const uint16_t* __restrict__ table, int size, float step,
                                                     uint16_t* __restrict__ out) {
  __shared__ float sh[32];
  const float* row = x + static_cast<int64_t>(blockIdx.x) * cols;
  uint16_t* orow = out + static_cast<int64_t>(blockIdx.x) * cols;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += 256) m = nanmax_f(m, row[c]);
  m = block_reduce_max<256>(m, sh);
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += 256) s += lut_exp(table, row[c] - m, step, size);
  s = block_reduce_sum<256>(s, sh);
  if (!(s > 0.0f)) s = 1.0f;  // zero-sum guard (attention.py:131)
  for (int64_t c = threadIdx.x; c < cols; c += 256)
    orow[c] = __half_as_ushort(__float2half_rn(__fdiv_rn(lut_exp(table, row[c] - m, step, size), s)));
}

// ---------------------------------------------------------------------------
// Decode attention
// ---------------------------------------------------------------------------
struct AttnWs {
  uint32_t* err;
  uint32_t* counters;  // [T*H]
  float* stats;        // [T*H][2]: row max, LUT sum
  float* cmax;         // [T*H][C]
  float* scores;       // [T*H][Lg]
  float* part;         // [T*H][C][d] fp32 per-chunk partial outputs
  // Optional per-trace lengths read on the device (a captured decode step replays with
  // a growing cache): L = min(Lg, lens[t] + len_add) for the rows of trace t = row / heads.
  const int32_t* lens;
  int len_add, heads;
};

// Valid key length of a (trace, head) row; Lg sizes the grid and the workspace.
__device__ __forceinline__ int attn_len(const AttnWs& w, int row, int Lg) {
  if (!w.lens) return Lg;
  return max(0, min(Lg, w.lens[row / w.heads] + w.len_add));
}

constexpr int kAttnBlock = 256;
constexpr int kAttnU = 8;  // score loads in flight per thread in the statistics pass

static inline int attn_chunks(int L) { return std::max(1, std::min(64, (L + 511) / 512)); }

// Pass 1: scores for one (trace, head) and one chunk of the KV length.
// A group of TPR = d / 8 threads owns TPR consecutive key rows per pass; each thread
// holds an 8-value slice of d and forms its partial dot product for all TPR rows, then
// a transposing butterfly (TPR - 1 shuffles for TPR rows) leaves thread `sub` with
// the full dot product of row `sub`.
template <int TPR>
__global__ void __launch_bounds__(kAttnBlock) k_attn_scores(const uint16_t* __restrict__ q,
                                                            const uint16_t* __restrict__ k, int Lg, int64_t kvs,
                                                            int C, float scale, AttnWs w) {
  constexpr int D = TPR * 8;
  constexpr int G = kAttnBlock / TPR;  // thread groups
  constexpr int B = TPR;  // key rows loaded per batch: a group's rows all in flight
  __shared__ float sh[32];
  const int row = blockIdx.y;  // t*H + h
  const int chunk = blockIdx.x;
  const int Lc = (Lg + C - 1) / C;
  const int sub = threadIdx.x % TPR, grp = threadIdx.x / TPR;
  // q and K may come from the previous kernel, and the workspace is still read by the
  // previous call's last pass: wait for it, then let the next pass launch
  pdl_wait();
  pdl_launch_dependents();
  const int L = attn_len(w, row, Lg);
  const int l0 = chunk * Lc, l1 = min(L, l0 + Lc);
  float qf[8];
  {
    const uint4 qv = *reinterpret_cast<const uint4*>(q + static_cast<int64_t>(row) * D + sub * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      qf[2 * i] = f.x;
      qf[2 * i + 1] = f.y;
    }
  }
  if (chunk == 0 && threadIdx.x == 0) w.counters[row] = 0u;  // pass 3's arrival counter
  const uint16_t* kb = k + static_cast<int64_t>(row) * kvs;
  float m = -INFINITY;
  for (int pbase = l0; pbase < l1; pbase += G * TPR) {  // uniform trip count: shuffles below
    const int base = pbase + grp * TPR;
    float v[TPR];
#pragma unroll
    for (int j0 = 0; j0 < TPR; j0 += B) {
      uint4 kv[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int l = base + j0 + b;
        kv[b] = l < l1 ? __ldcs(reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(l) * D + sub * 8))
                       : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const __half2* h = reinterpret_cast<const __half2*>(&kv[b]);
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          dot = fmaf(qf[2 * i], f.x, dot);
          dot = fmaf(qf[2 * i + 1], f.y, dot);
        }
        v[j0 + b] = dot;
      }
    }
    // butterfly: at width s, lanes with bit s set keep rows j + s, the others rows j
#pragma unroll
    for (int s = TPR / 2; s >= 1; s >>= 1) {
      const bool up = (sub & s) != 0;
#pragma unroll
      for (int j = 0; j < s; ++j) {
        const float send = up ? v[j] : v[j + s];
        const float keep = up ? v[j + s] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
      }
    }
    const int l = base + sub;
    if (l < l1) {
      const float sc = v[0] * scale;
      w.scores[static_cast<int64_t>(row) * Lg + l] = sc;
      m = nanmax_f(m, sc);
    }
  }
  m = block_reduce_max<kAttnBlock>(m, sh);
  if (threadIdx.x == 0) w.cmax[static_cast<int64_t>(row) * C + chunk] = m;
}

// Pass 2: row max over the chunk maxima, fp32 sum of the LUT values.
__global__ void __launch_bounds__(kAttnBlock) k_attn_stats(int Lg, int C, const uint16_t* __restrict__ table, int size,
                                                           float step, AttnWs w) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  pdl_wait();  // the scores pass has finished
  pdl_launch_dependents();
  const int L = attn_len(w, row, Lg);
  float m = -INFINITY;
  for (int c = threadIdx.x; c < C; c += kAttnBlock) m = nanmax_f(m, w.cmax[static_cast<int64_t>(row) * C + c]);
  m = block_reduce_max<kAttnBlock>(m, sh);
  const float* s = w.scores + static_cast<int64_t>(row) * Lg;
  float acc = 0.0f;
  for (int l0 = threadIdx.x; l0 < L; l0 += kAttnBlock * kAttnU) {  // kAttnU loads in flight, summed in order
    float x[kAttnU];
#pragma unroll
    for (int u = 0; u < kAttnU; ++u) {
      const int l = l0 + u * kAttnBlock;
      x[u] = l < L ? __ldcg(s + l) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kAttnU; ++u)
      if (l0 + u * kAttnBlock < L) acc += lut_exp(table, x[u] - m, step, size);
  }
  acc = block_reduce_sum<kAttnBlock>(acc, sh);
  if (threadIdx.x == 0) {
    w.stats[2 * row] = m;
    w.stats[2 * row + 1] = (acc > 0.0f) ? acc : 1.0f;
  }
}

// Pass 3: out = sum_l fp16(LUT(s_l - m) / sum) * v_l, one chunk per CTA. A group of
// TPR threads owns TPR consecutive rows per pass: thread `sub` forms the probability of
// row `sub` once, and a shuffle hands it to the group for that row's products.
template <int TPR>
__global__ void __launch_bounds__(kAttnBlock) k_attn_pv(const uint16_t* __restrict__ v, uint16_t* __restrict__ out,
                                                        int Lg, int64_t kvs, int C, const uint16_t* __restrict__ table,
                                                        int size, float step, AttnWs w) {
  constexpr int D = TPR * 8;
  constexpr int G = kAttnBlock / TPR;
  constexpr int B = TPR < 8 ? TPR : 8;
  __shared__ float red[kAttnBlock * 8];
  __shared__ int is_last;
  const int row = blockIdx.y, chunk = blockIdx.x;
  const int Lc = (Lg + C - 1) / C;
  // the lengths array is not written by the passes of this call: readable before the wait
  const int L = attn_len(w, row, Lg);
  const int l0 = chunk * Lc, l1 = min(L, l0 + Lc);
  const int sub = threadIdx.x % TPR, grp = threadIdx.x / TPR;
  const uint16_t* vb = v + static_cast<int64_t>(row) * kvs;
  // Every kernel of this path lets its successor launch only after its own wait, so
  // when this one starts, the kernel before the scores pass (the producer of V) has
  // finished: V of the first pass can be pulled into L2 while the statistics pass runs.
  for (int l = l0 + threadIdx.x / (D / 64 > 0 ? D / 64 : 1); l < min(l1, l0 + G * TPR);
       l += kAttnBlock / (D / 64 > 0 ? D / 64 : 1)) {
    const int part = D >= 64 ? threadIdx.x % (D / 64) : 0;  // 128-byte lines of a row
    asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + static_cast<int64_t>(l) * D + part * 64));
  }
  pdl_wait();  // the statistics pass has finished
  pdl_launch_dependents();
  const float m = w.stats[2 * row], sum = w.stats[2 * row + 1];
  const float* s = w.scores + static_cast<int64_t>(row) * Lg;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int pbase = l0; pbase < l1; pbase += G * TPR) {  // uniform trip count: shuffles below
    const int base = pbase + grp * TPR;
    float p = 0.0f;
    if (base + sub < l1) {
      const float e = lut_exp(table, __ldcg(s + base + sub) - m, step, size);
      p = __half2float(__float2half_rn(__fdiv_rn(e, sum)));
    }
#pragma unroll
    for (int j0 = 0; j0 < TPR; j0 += B) {
      uint4 vv[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int l = base + j0 + b;
        vv[b] = l < l1 ? __ldcs(reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(l) * D + sub * 8))
                       : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float pj = __shfl_sync(0xffffffffu, p, j0 + b, TPR);  // zero past l1
        const __half2* h = reinterpret_cast<const __half2*>(&vv[b]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          acc[2 * i] = fmaf(pj, f.x, acc[2 * i]);
          acc[2 * i + 1] = fmaf(pj, f.y, acc[2 * i + 1]);
        }
      }
    }
  }
  // reduce across the row groups (fixed order): red[grp][D]
#pragma unroll
  for (int i = 0; i < 8; ++i) red[threadIdx.x * 8 + i] = acc[i];  // index = (grp*TPR+sub)*8+i
  __syncthreads();
  float* part = w.part + static_cast<int64_t>(row) * C * D;
  for (int dd = threadIdx.x; dd < D; dd += kAttnBlock) {
    float t = 0.0f;
    for (int g = 0; g < G; ++g) t += red[g * D + dd];
    __stcg(part + static_cast<int64_t>(chunk) * D + dd, t);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(&w.counters[row], 1u) == static_cast<uint32_t>(C - 1));
  __syncthreads();
  if (is_last) {  // the last chunk sums all chunks in chunk order: deterministic
    __threadfence();
    for (int dd = threadIdx.x; dd < D; dd += kAttnBlock) {
      float t = 0.0f;
      for (int c = 0; c < C; ++c) t += __ldcg(part + static_cast<int64_t>(c) * D + dd);
      out[static_cast<int64_t>(row) * D + dd] = __half_as_ushort(__float2half_rn(t));
    }
  }
}

// All three passes in one CTA per (trace, head) row, for caches short enough that a
// row's scores fit in shared memory (at most kAttnFusedMax positions): the scores pass
// of k_attn_scores into shared memory, the row max and LUT sum of k_attn_stats, and
// the P·V pass of k_attn_pv over the whole row, with the same per-element arithmetic.
// One launch and no cross-CTA merge; the split passes keep long caches, whose rows
// need many CTAs each to fill the GPU.
constexpr int kAttnFusedMax = 2048;

template <int TPR>
__global__ void __launch_bounds__(kAttnBlock) k_attn_fused(const uint16_t* __restrict__ q,
                                                           const uint16_t* __restrict__ k,
                                                           const uint16_t* __restrict__ v, uint16_t* __restrict__ out,
                                                           int Lg, int64_t kvs, float scale,
                                                           const uint16_t* __restrict__ table, int size, float step,
                                                           AttnWs w) {
  constexpr int D = TPR * 8;
  constexpr int G = kAttnBlock / TPR;
  __shared__ float sh[32];
  __shared__ float red[kAttnBlock * 8];
  extern __shared__ float sc[];  // [Lg] scores of this row
  const int row = blockIdx.x;
  const int sub = threadIdx.x % TPR, grp = threadIdx.x / TPR;
  pdl_wait();  // q, K and V may come from the previous kernel
  pdl_launch_dependents();
  const int L = attn_len(w, row, Lg);
  float qf[8];
  {
    const uint4 qv = *reinterpret_cast<const uint4*>(q + static_cast<int64_t>(row) * D + sub * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      qf[2 * i] = f.x;
      qf[2 * i + 1] = f.y;
    }
  }
  const uint16_t* kb = k + static_cast<int64_t>(row) * kvs;
  const uint16_t* vb = v + static_cast<int64_t>(row) * kvs;
  // scores: a group owns TPR consecutive rows per pass (butterfly as in k_attn_scores)
  float m = -INFINITY;
  for (int pbase = 0; pbase < L; pbase += G * TPR) {
    const int base = pbase + grp * TPR;
    float vv[TPR];
    {
      uint4 kv[TPR];
#pragma unroll
      for (int b = 0; b < TPR; ++b) {
        const int l = base + b;
        kv[b] = l < L ? __ldcs(reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(l) * D + sub * 8))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int b = 0; b < TPR; ++b) {
        const __half2* h = reinterpret_cast<const __half2*>(&kv[b]);
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          dot = fmaf(qf[2 * i], f.x, dot);
          dot = fmaf(qf[2 * i + 1], f.y, dot);
        }
        vv[b] = dot;
      }
    }
#pragma unroll
    for (int s = TPR / 2; s >= 1; s >>= 1) {
      const bool up = (sub & s) != 0;
#pragma unroll
      for (int j = 0; j < s; ++j) {
        const float send = up ? vv[j] : vv[j + s];
        const float keep = up ? vv[j + s] : vv[j];
        vv[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
      }
    }
    const int l = base + sub;
    if (l < L) {
      const float x = vv[0] * scale;
      sc[l] = x;
      m = nanmax_f(m, x);
    }
  }
  m = block_reduce_max<kAttnBlock>(m, sh);  // synchronises: all scores are in sc[]
  // LUT sum in the order of k_attn_stats (per thread l = t, t + block, ..., then the block)
  float acc = 0.0f;
  for (int l = threadIdx.x; l < L; l += kAttnBlock) acc += lut_exp(table, sc[l] - m, step, size);
  acc = block_reduce_sum<kAttnBlock>(acc, sh);
  const float sum = acc > 0.0f ? acc : 1.0f;
  // P·V over the whole row
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.0f;
  for (int pbase = 0; pbase < L; pbase += G * TPR) {
    const int base = pbase + grp * TPR;
    float p = 0.0f;
    if (base + sub < L) {
      const float e = lut_exp(table, sc[base + sub] - m, step, size);
      p = __half2float(__float2half_rn(__fdiv_rn(e, sum)));
    }
    uint4 vr[TPR];
#pragma unroll
    for (int b = 0; b < TPR; ++b) {
      const int l = base + b;
      vr[b] = l < L ? __ldcs(reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(l) * D + sub * 8))
                    : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int b = 0; b < TPR; ++b) {
      const float pj = __shfl_sync(0xffffffffu, p, b, TPR);  // zero past L
      const __half2* h = reinterpret_cast<const __half2*>(&vr[b]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        o[2 * i] = fmaf(pj, f.x, o[2 * i]);
        o[2 * i + 1] = fmaf(pj, f.y, o[2 * i + 1]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[threadIdx.x * 8 + i] = o[i];  // index = (grp*TPR+sub)*8+i
  __syncthreads();
  for (int dd = threadIdx.x; dd < D; dd += kAttnBlock) {
    float t = 0.0f;
    for (int g = 0; g < G; ++g) t += red[g * D + dd];
    out[static_cast<int64_t>(row) * D + dd] = __half_as_ushort(__float2half_rn(t));
  }
}

// ---------------------------------------------------------------------------
// Streaming path for rows of up to kAttnStreamMax keys (the decode step's caches):
// one CTA per (trace, head) row, no workspace, one launch. A producer warp streams the
// row's K rows and then its V rows through a ring of kStrRing shared-memory stages with
// bulk copies (cp.async.bulk, no multicast, completion on mbarriers), so the V stream
// starts while the last scores are formed and the memory system always holds a full
// ring of this row's requests. Eight consumer warps:
//   1. scores of every K stage -> shared memory (16-byte slices of a key per lane,
//      xor-shuffle sum over the d / 8 lanes of a key), row max;
//   2. e_l = LUT(s_l - max) in place and their sum (the strided-then-block order of
//      k_attn_stats), then p_l = fp16(e_l / sum) in place;
//   3. P.V over every V stage as it lands, fp32; per-warp partials summed in warp order.
// Per element the arithmetic is that of the split passes; the order of the output sum
// differs. Deterministic.
// ---------------------------------------------------------------------------
constexpr int kAttnStreamMax = 2048;  // keys per row held as scores in shared memory
constexpr int kStrWarps = 8;          // consumer warps
constexpr int kStrStage = 32768;      // bytes per ring stage
constexpr int kStrRing = 3;           // ring stages

__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4u(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// Block reductions over the consumer warps only (named barrier 1; the producer warp
// takes no part).
__device__ __forceinline__ float cons_reduce(float v, float* sh, bool is_max) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? nanmax_f(v, u) : v + u;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  named_bar_sync(1, kStrWarps * 32);
  if (l == 0) sh[w] = v;
  named_bar_sync(1, kStrWarps * 32);
  v = sh[0];
  for (int i = 1; i < kStrWarps; ++i) v = is_max ? nanmax_f(v, sh[i]) : v + sh[i];
  return v;
}

template <int TPR>
__global__ void __launch_bounds__((kStrWarps + 1) * 32) k_attn_stream(const uint16_t* __restrict__ q,
                                                                      const uint16_t* __restrict__ k,
                                                                      const uint16_t* __restrict__ v,
                                                                      uint16_t* __restrict__ out, int Lg, int64_t kvs,
                                                                      float scale, const uint16_t* __restrict__ table,
                                                                      int size, float step, AttnWs w) {
  constexpr int D = TPR * 8;
  constexpr int KS = kStrStage / (D * 2);  // keys per stage
  constexpr int KW = 32 / TPR;             // keys per warp step
  constexpr int IT = KS / (kStrWarps * KW);  // warp steps per stage (8 for every d)
  constexpr int CT = kStrWarps * 32;
  static_assert(IT * kStrWarps * KW == KS, "stage split");
  extern __shared__ __align__(128) uint8_t dyn[];
  uint8_t* ring = dyn;                                                   // [kStrRing][kStrStage]
  float* sc = reinterpret_cast<float*>(dyn + kStrRing * kStrStage);      // [Lg]
  float* red = sc + ((Lg + 3) & ~3);                                     // [kStrWarps][D]
  __shared__ __align__(8) uint64_t full[kStrRing], empty[kStrRing];
  __shared__ float sh[kStrWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int r = 0; r < kStrRing; ++r) {
      mbar_init(full + r, 1);
      mbar_init(empty + r, kStrWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // q, K, V and the lengths may come from the previous kernel
  pdl_launch_dependents();
  const int L = attn_len(w, row, Lg);
  const int nK = (L + KS - 1) / KS;  // K stages, then as many V stages
  if (warp == kStrWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();  // every cache byte is read once per call
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(k + static_cast<int64_t>(row) * kvs);
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(v + static_cast<int64_t>(row) * kvs);
      for (int s = 0; s < 2 * nK; ++s) {
        const int slot = s % kStrRing;
        if (s >= kStrRing && !mbar_wait(empty + slot, ((s / kStrRing) - 1) & 1) && w.err)
          atomicOr(w.err, MB_DEVERR_TIMEOUT);
        const int kk = s < nK ? s : s - nK;
        const uint32_t bytes = static_cast<uint32_t>(min(KS, L - kk * KS)) * D * 2;
        mbar_expect_tx(full + slot, bytes);
        bulk_load_g2s(ring + slot * kStrStage, (s < nK ? kb : vb) + static_cast<size_t>(kk) * KS * D * 2, bytes,
                      full + slot, pol);
      }
    }
    return;
  }
  // ---------------- consumers ----------------
  const int sub = lane % TPR, ks = lane / TPR;  // 16-byte slice of d, key slot of the warp step
  float qf[8];
  {
    const uint4 qv = *reinterpret_cast<const uint4*>(q + static_cast<int64_t>(row) * D + sub * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      qf[2 * i] = f.x;
      qf[2 * i + 1] = f.y;
    }
  }
  float m = -INFINITY;
  for (int s = 0; s < nK; ++s) {
    const int slot = s % kStrRing;
    if (!mbar_wait(full + slot, (s / kStrRing) & 1) && lane == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
    const int j0 = s * KS, rows = min(KS, L - j0);
    const uint8_t* st = ring + slot * kStrStage;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int kr = (it * kStrWarps + warp) * KW + ks;
      float dot = 0.0f;
      if (kr < rows) {
        const uint4 kv = ld_shared_v4u(st + kr * D * 2 + sub * 16);
        const __half2* h = reinterpret_cast<const __half2*>(&kv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          dot = fmaf(qf[2 * i], f.x, dot);
          dot = fmaf(qf[2 * i + 1], f.y, dot);
        }
      }
#pragma unroll
      for (int o = TPR / 2; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (sub == 0 && kr < rows) {
        const float x = dot * scale;
        sc[j0 + kr] = x;
        m = nanmax_f(m, x);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }
  m = cons_reduce(m, sh, true);  // every score is in sc[]
  float acc = 0.0f;
  for (int j = threadIdx.x; j < L; j += CT) {
    const float e = lut_exp(table, sc[j] - m, step, size);
    sc[j] = e;
    acc += e;
  }
  acc = cons_reduce(acc, sh, false);
  const float sum = acc > 0.0f ? acc : 1.0f;
  for (int j = threadIdx.x; j < L; j += CT) sc[j] = __half2float(__float2half_rn(__fdiv_rn(sc[j], sum)));
  named_bar_sync(1, CT);  // every p_l is in sc[]
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.0f;
  for (int s = nK; s < 2 * nK; ++s) {
    const int slot = s % kStrRing;
    if (!mbar_wait(full + slot, (s / kStrRing) & 1) && lane == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
    const int j0 = (s - nK) * KS, rows = min(KS, L - j0);
    const uint8_t* st = ring + slot * kStrStage;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int kr = (it * kStrWarps + warp) * KW + ks;
      if (kr < rows) {
        const float p = sc[j0 + kr];
        const uint4 vv = ld_shared_v4u(st + kr * D * 2 + sub * 16);
        const __half2* h = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          o[2 * i] = fmaf(p, f.x, o[2 * i]);
          o[2 * i + 1] = fmaf(p, f.y, o[2 * i + 1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }
  // the KW key slots of a warp hold the same slice of d: sum them, then the warps
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int x = TPR; x < 32; x <<= 1) o[i] += __shfl_xor_sync(0xffffffffu, o[i], x);
  if (ks == 0)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * D + sub * 8 + i] = o[i];
  named_bar_sync(1, CT);
  for (int dd = threadIdx.x; dd < D; dd += CT) {
    float t = 0.0f;
    for (int g = 0; g < kStrWarps; ++g) t += red[g * D + dd];
    out[static_cast<int64_t>(row) * D + dd] = __half_as_ushort(__float2half_rn(t));
  }
}

// Split form for few rows (fewer than the SMs, e.g. a tensor-parallel rank's heads):
// one cluster of S CTAs per row, CTA c streaming the keys [c * per, (c + 1) * per) of
// the row's valid length through its own ring exactly as k_attn_stream does, so a row
// moves at S CTAs' rate. The row max, the LUT sum and the partial outputs are joined
// through distributed shared memory: a CTA stores its value into a slot of every CTA
// (the outputs only into the leader's) and arrives on that CTA's mbarrier (release,
// cluster scope); a CTA reads the slots once its own mbarrier has seen all S arrivals
// (acquire, bounded wait). The only cluster barrier is the one after the mbarriers are
// initialised, which every thread passes before the producer warp splits off. Same
// per-element arithmetic as k_attn_stream; the sums run over the S CTAs in order.
constexpr int kAttnSplitMax = 8;  // portable cluster size

__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const long long t0 = clock64();
  while (!try_once())
    if (clock64() - t0 > kWaitBudget) return false;
  return true;
}

template <int TPR>
__global__ void __launch_bounds__((kStrWarps + 1) * 32) k_attn_stream_split(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
    uint16_t* __restrict__ out, int Lg, int64_t kvs, int Lc, float scale, const uint16_t* __restrict__ table,
    int size, float step, AttnWs w) {
  constexpr int D = TPR * 8;
  constexpr int KS = kStrStage / (D * 2);
  constexpr int KW = 32 / TPR;
  constexpr int IT = KS / (kStrWarps * KW);
  constexpr int CT = kStrWarps * 32;
  extern __shared__ __align__(128) uint8_t dyn[];
  uint8_t* ring = dyn;                                               // [kStrRing][kStrStage]
  float* sc = reinterpret_cast<float*>(dyn + kStrRing * kStrStage);  // [Lc]
  float* red = sc + ((Lc + 3) & ~3);                                 // [kStrWarps][D]
  float* xpart = red + kStrWarps * D;                                // [S][D]: the leader's slots
  __shared__ __align__(8) uint64_t full[kStrRing], empty[kStrRing], xbar[3];
  __shared__ float sh[kStrWarps];
  __shared__ float xmax[kAttnSplitMax], xsum[kAttnSplitMax];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = static_cast<int>(gridDim.x);  // cluster dims (S, 1, 1)
  const int c = static_cast<int>(cluster_ctarank());
  const int row = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int r = 0; r < kStrRing; ++r) {
      mbar_init(full + r, 1);
      mbar_init(empty + r, kStrWarps);
    }
    for (int i = 0; i < 3; ++i) mbar_init(xbar + i, S);  // one arrival per CTA of the cluster
    fence_mbar_init();
  }
  cluster_sync();  // every CTA's mbarriers exist before anyone arrives on them remotely
  pdl_wait();      // q, K, V and the lengths may come from the previous kernel
  pdl_launch_dependents();
  const int L = attn_len(w, row, Lg);
  const int per = ((L + S - 1) / S + 15) & ~15;  // <= Lc: the host sized Lc for Lg >= L
  const int l0 = min(L, c * per);
  const int n = min(L, l0 + per) - l0;  // this CTA's keys
  const int nK = (n + KS - 1) / KS;
  if (warp == kStrWarps) {
    // ---------------- producer: this CTA's K rows, then its V rows ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(k + static_cast<int64_t>(row) * kvs + static_cast<int64_t>(l0) * D);
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(v + static_cast<int64_t>(row) * kvs + static_cast<int64_t>(l0) * D);
      for (int s = 0; s < 2 * nK; ++s) {
        const int slot = s % kStrRing;
        if (s >= kStrRing && !mbar_wait(empty + slot, ((s / kStrRing) - 1) & 1) && w.err)
          atomicOr(w.err, MB_DEVERR_TIMEOUT);
        const int kk = s < nK ? s : s - nK;
        const uint32_t bytes = static_cast<uint32_t>(min(KS, n - kk * KS)) * D * 2;
        mbar_expect_tx(full + slot, bytes);
        bulk_load_g2s(ring + slot * kStrStage, (s < nK ? kb : vb) + static_cast<size_t>(kk) * KS * D * 2, bytes,
                      full + slot, pol);
      }
    }
    return;
  }
  // ---------------- consumers ----------------
  const int sub = lane % TPR, ks = lane / TPR;
  float qf[8];
  {
    const uint4 qv = *reinterpret_cast<const uint4*>(q + static_cast<int64_t>(row) * D + sub * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      qf[2 * i] = f.x;
      qf[2 * i + 1] = f.y;
    }
  }
  float m = -INFINITY;
  for (int s = 0; s < nK; ++s) {
    const int slot = s % kStrRing;
    if (!mbar_wait(full + slot, (s / kStrRing) & 1) && lane == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
    const int j0 = s * KS, rows = min(KS, n - j0);
    const uint8_t* st = ring + slot * kStrStage;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int kr = (it * kStrWarps + warp) * KW + ks;
      float dot = 0.0f;
      if (kr < rows) {
        const uint4 kv = ld_shared_v4u(st + kr * D * 2 + sub * 16);
        const __half2* h = reinterpret_cast<const __half2*>(&kv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          dot = fmaf(qf[2 * i], f.x, dot);
          dot = fmaf(qf[2 * i + 1], f.y, dot);
        }
      }
#pragma unroll
      for (int o = TPR / 2; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (sub == 0 && kr < rows) {
        const float x = dot * scale;
        sc[j0 + kr] = x;
        m = nanmax_f(m, x);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }
  m = cons_reduce(m, sh, true);
  // row max: this CTA's max into slot c of every CTA, then wait for all S
  if (threadIdx.x < S) {
    st_shared_cluster_f32(mapa_shared(smem_u32(&xmax[c]), threadIdx.x), m);
    mbar_arrive_remote(mapa_shared(smem_u32(&xbar[0]), threadIdx.x));
  }
  if (!mbar_wait_cluster(&xbar[0], 0) && threadIdx.x == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
  float gm = -INFINITY;
  for (int i = 0; i < S; ++i) gm = nanmax_f(gm, xmax[i]);
  float acc = 0.0f;
  for (int j = threadIdx.x; j < n; j += CT) {
    const float e = lut_exp(table, sc[j] - gm, step, size);
    sc[j] = e;
    acc += e;
  }
  acc = cons_reduce(acc, sh, false);
  if (threadIdx.x < S) {
    st_shared_cluster_f32(mapa_shared(smem_u32(&xsum[c]), threadIdx.x), acc);
    mbar_arrive_remote(mapa_shared(smem_u32(&xbar[1]), threadIdx.x));
  }
  if (!mbar_wait_cluster(&xbar[1], 0) && threadIdx.x == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
  float tot = 0.0f;
  for (int i = 0; i < S; ++i) tot += xsum[i];
  const float sum = tot > 0.0f ? tot : 1.0f;
  for (int j = threadIdx.x; j < n; j += CT) sc[j] = __half2float(__float2half_rn(__fdiv_rn(sc[j], sum)));
  named_bar_sync(1, CT);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.0f;
  for (int s = nK; s < 2 * nK; ++s) {
    const int slot = s % kStrRing;
    if (!mbar_wait(full + slot, (s / kStrRing) & 1) && lane == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
    const int j0 = (s - nK) * KS, rows = min(KS, n - j0);
    const uint8_t* st = ring + slot * kStrStage;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int kr = (it * kStrWarps + warp) * KW + ks;
      if (kr < rows) {
        const float p = sc[j0 + kr];
        const uint4 vv = ld_shared_v4u(st + kr * D * 2 + sub * 16);
        const __half2* h = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          o[2 * i] = fmaf(p, f.x, o[2 * i]);
          o[2 * i + 1] = fmaf(p, f.y, o[2 * i + 1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int x = TPR; x < 32; x <<= 1) o[i] += __shfl_xor_sync(0xffffffffu, o[i], x);
  if (ks == 0)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * D + sub * 8 + i] = o[i];
  named_bar_sync(1, CT);
  // this CTA's partial output into the leader's slot c, then one arrival there (the
  // barrier above orders every thread's stores before thread 0's release)
  for (int dd = threadIdx.x; dd < D; dd += CT) {
    float t = 0.0f;
    for (int g = 0; g < kStrWarps; ++g) t += red[g * D + dd];
    st_shared_cluster_f32(mapa_shared(smem_u32(&xpart[c * D + dd]), 0), t);
  }
  if (threadIdx.x < D) asm volatile("fence.acq_rel.cluster;" ::: "memory");  // visible cluster-wide
  named_bar_sync(1, CT);
  if (threadIdx.x == 0) mbar_arrive_remote(mapa_shared(smem_u32(&xbar[2]), 0));
  if (c == 0) {
    if (!mbar_wait_cluster(&xbar[2], 0) && threadIdx.x == 0 && w.err) atomicOr(w.err, MB_DEVERR_TIMEOUT);
    for (int dd = threadIdx.x; dd < D; dd += CT) {
      float t = 0.0f;
      for (int i = 0; i < S; ++i) t += xpart[i * D + dd];
      out[static_cast<int64_t>(row) * D + dd] = __half_as_ushort(__float2half_rn(t));
    }
  }
}

// Split size for `rows` rows of up to Lg keys: about two CTAs per SM in all, at most
// kAttnSplitMax, at least 16 keys each; 1 = the one-CTA-per-row kernel.
static int attn_split(int rows, int Lg) {
  if (rows >= 148) return 1;
  return std::max(1, std::min({kAttnSplitMax, (2 * 148) / rows, (Lg + 15) / 16}));
}

static size_t attn_split_smem(int Lg, int d, int S) {
  const int Lc = ((Lg + S - 1) / S + 15) & ~15;
  return static_cast<size_t>(kStrRing) * kStrStage + static_cast<size_t>((Lc + 3) & ~3) * 4 +
         static_cast<size_t>(kStrWarps) * d * 4 + static_cast<size_t>(S) * d * 4;
}

static size_t attn_stream_smem(int Lg, int d) {
  return static_cast<size_t>(kStrRing) * kStrStage + static_cast<size_t>((Lg + 3) & ~3) * 4 +
         static_cast<size_t>(kStrWarps) * d * 4;
}

static inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

static AttnWs carve_attn_ws(void* base, int T, int H, int L, int d, int C, size_t* total) {
  const size_t rows = static_cast<size_t>(T) * H;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  AttnWs w;
  w.err = reinterpret_cast<uint32_t*>(p + off);
  off += 256;
  w.counters = reinterpret_cast<uint32_t*>(p + off);
  off += align256(rows * 4);
  w.stats = reinterpret_cast<float*>(p + off);
  off += align256(rows * 8);
  w.cmax = reinterpret_cast<float*>(p + off);
  off += align256(rows * C * 4);
  w.part = reinterpret_cast<float*>(p + off);
  off += align256(rows * C * d * 4);
  w.scores = reinterpret_cast<float*>(p + off);
  off += align256(rows * static_cast<size_t>(L) * 4);
  w.lens = nullptr;
  w.len_add = 0;
  w.heads = H;
  if (total) *total = off;
  return w;
}

// The three passes of mb_decode_attn over a scratch base that holds at least
// mb_decode_attn_workspace_size(T, H, L, d) bytes, 256-byte aligned; arguments
// already validated by the caller. Used by the fixed-scratch entry point
// (attention_noalloc.cu).
// Launch with programmatic dependent launch: the kernel may start while its
// predecessor on the stream finishes; it waits (griddepcontrol.wait) before touching
// anything the predecessor writes.
template <typename Kern, typename... Args>
static int launch_pdl_smem(Kern kern, dim3 grid, cudaStream_t st, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnBlock);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

template <typename Kern, typename... Args>
static int launch_pdl(Kern kern, dim3 grid, cudaStream_t st, Args... args) {
  return launch_pdl_smem(kern, grid, st, 0, args...);
}

template <int TPR>
static int32_t attn_launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int L, int64_t kvs,
                           int C, int rows, float scale, const uint16_t* table, int size, float step, const AttnWs& w,
                           cudaStream_t st) {
  if (L <= kAttnFusedMax) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0;
    const int S = attn_split(rows, L);
    if (aligned && L <= kAttnStreamMax && S > 1 && rows <= 65535) {  // few rows: S CTAs per row
      const size_t smem = attn_split_smem(L, TPR * 8, S);
      if (cudaFuncSetAttribute(k_attn_stream_split<TPR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return MB_ERR_LAUNCH;
      const int Lc = ((L + S - 1) / S + 15) & ~15;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S, rows);
      cfg.blockDim = dim3((kStrWarps + 1) * 32);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = S;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      if (cudaLaunchKernelEx(&cfg, k_attn_stream_split<TPR>, q, k, v, out, L, kvs, Lc, scale, table, size, step, w) !=
          cudaSuccess) {
        (void)cudaGetLastError();
        return MB_ERR_LAUNCH;
      }
      return MB_OK;
    }
    if (aligned && L <= kAttnStreamMax) {  // kvs * 2 bytes is a multiple of 16 for every d >= 8
      const size_t smem = attn_stream_smem(L, TPR * 8);
      if (cudaFuncSetAttribute(k_attn_stream<TPR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return MB_ERR_LAUNCH;
      return launch_with_pdl(k_attn_stream<TPR>, dim3(rows), dim3((kStrWarps + 1) * 32), smem, st, q, k, v, out, L,
                             kvs, scale, table, size, step, w);
    }
    // one CTA per row, scores in shared memory
    const int smem = L * 4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k_attn_fused<TPR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return MB_ERR_LAUNCH;
    return launch_pdl_smem(k_attn_fused<TPR>, dim3(rows), st, static_cast<size_t>(smem), q, k, v, out, L, kvs,
                           scale, table, size, step, w);
  }
  if (launch_pdl(k_attn_scores<TPR>, dim3(C, rows), st, q, k, L, kvs, C, scale, w) != MB_OK) return MB_ERR_LAUNCH;
  if (launch_pdl(k_attn_stats, dim3(rows), st, L, C, table, size, step, w) != MB_OK) return MB_ERR_LAUNCH;
  if (launch_pdl(k_attn_pv<TPR>, dim3(C, rows), st, v, out, L, kvs, C, table, size, step, w) != MB_OK)
    return MB_ERR_LAUNCH;
  return MB_OK;
}

// The three passes of mb_decode_attn over a scratch base that holds at least
// mb_decode_attn_workspace_size(T, H, L, d) bytes, 256-byte aligned; arguments
// already validated by the caller (d a power of two in [8, 256]). kv_stride: elements
// between the K (and V) rows of consecutive (trace, head) pairs; 0 = L * d (packed).
// lens (optional, device): per-trace lengths, the valid length of trace t being
// min(L, lens[t] + len_add); L then sizes the grid and the workspace.
int32_t decode_attn_enqueue(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int T, int H,
                            int L, int d, float scale, const uint16_t* table, int size, float range_max,
                            void* scratch, cudaStream_t st, int64_t kv_stride, const int32_t* lens,
                            int len_add) {
  const int C = attn_chunks(L);
  AttnWs w = carve_attn_ws(scratch, T, H, L, d, C, nullptr);
  w.lens = lens;
  w.len_add = len_add;
  const float step = static_cast<float>(static_cast<double>(range_max) / (size - 1));
  const int rows = T * H;
  const int64_t kvs = kv_stride > 0 ? kv_stride : static_cast<int64_t>(L) * d;
  switch (d) {
    case 8: return attn_launch<1>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    case 16: return attn_launch<2>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    case 32: return attn_launch<4>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    case 64: return attn_launch<8>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    case 128: return attn_launch<16>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    case 256: return attn_launch<32>(q, k, v, out, L, kvs, C, rows, scale, table, size, step, w, st);
    default: return MB_ERR_ARGS;
  }
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_exp_lut_lookup(const uint16_t* table, int32_t size, float range_max, const float* x, int64_t n,
                          uint16_t* out, void* stream) {
  if (size < 2 || !(range_max > 0.0f) || n < 0) return MB_ERR_ARGS;
  if (n == 0) return MB_OK;
  if (!table || !x || !out) return MB_ERR_NULL;
  const float step = static_cast<float>(static_cast<double>(range_max) / (size - 1));
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sm_count()) * 32);
  k_lut_lookup<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(table, size, step, x, n, out);
  return launch_status();
}

int32_t mb_lut_softmax(const float* x, int64_t rows, int64_t cols, const uint16_t* table, int32_t size,
                       float range_max, uint16_t* out, void* stream) {
  if (!x || !table || !out) return MB_ERR_NULL;
  if (rows < 0 || cols < 1 || size < 2 || !(range_max > 0.0f) || rows > 2147483647LL) return MB_ERR_ARGS;
  if (rows == 0) return MB_OK;
  const float step = static_cast<float>(static_cast<double>(range_max) / (size - 1));
  k_lut_softmax<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, cols, table, size,
                                                                                           step, out);
  return launch_status();
}

size_t mb_decode_attn_workspace_size(int32_t T, int32_t H, int32_t L, int32_t d) {
  if (T < 1 || H < 1 || L < 1 || d < 1) return 0;
  size_t total = 0;
  carve_attn_ws(nullptr, T, H, L, d, attn_chunks(L), &total);
  return total;
}

int32_t mb_decode_attn(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int32_t T, int32_t H,
                       int32_t L, int32_t d, float scale, const uint16_t* table, int32_t size, float range_max,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out || !table || !workspace) return MB_ERR_NULL;
  if (T < 1 || H < 1 || L < 1 || d < 8 || d > 256 || d % 8 != 0 || (d & (d - 1)) != 0 || size < 2 ||
      !(range_max > 0.0f))
    return MB_ERR_ARGS;
  if (static_cast<int64_t>(T) * H > 65535) return MB_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(workspace, 256)) return MB_ERR_ALIGN;
  if (workspace_bytes < mb_decode_attn_workspace_size(T, H, L, d)) return MB_ERR_WORKSPACE;
  return decode_attn_enqueue(q, k, v, out, T, H, L, d, scale, table, size, range_max, workspace,
                             static_cast<cudaStream_t>(stream), 0, nullptr, 0);
}

int32_t mb_decode_attn_cache(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
                             int32_t T, int32_t H, int32_t L, int32_t Lmax, int32_t d, float scale,
                             const uint16_t* table, int32_t size, float range_max, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out || !table || !workspace) return MB_ERR_NULL;
  if (T < 1 || H < 1 || L < 1 || Lmax < L || d < 8 || d > 256 || (d & (d - 1)) != 0 || size < 2 ||
      !(range_max > 0.0f))
    return MB_ERR_ARGS;
  if (static_cast<int64_t>(T) * H > 65535) return MB_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 256))
    return MB_ERR_ALIGN;
  if (workspace_bytes < mb_decode_attn_workspace_size(T, H, L, d)) return MB_ERR_WORKSPACE;
  return decode_attn_enqueue(q, k_cache, v_cache, out, T, H, L, d, scale, table, size, range_max, workspace,
                             static_cast<cudaStream_t>(stream), static_cast<int64_t>(Lmax) * d, nullptr, 0);
}

int32_t mb_decode_attn_cache_lens(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
                                  int32_t T, int32_t H, int32_t Lmax, int32_t d, const int32_t* lens, int32_t len_add,
                                  float scale, const uint16_t* table, int32_t size, float range_max, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out || !table || !workspace || !lens) return MB_ERR_NULL;
  if (T < 1 || H < 1 || Lmax < 1 || d < 8 || d > 256 || (d & (d - 1)) != 0 || size < 2 || !(range_max > 0.0f))
    return MB_ERR_ARGS;
  if (static_cast<int64_t>(T) * H > 65535) return MB_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 256))
    return MB_ERR_ALIGN;
  if (workspace_bytes < mb_decode_attn_workspace_size(T, H, Lmax, d)) return MB_ERR_WORKSPACE;
  return decode_attn_enqueue(q, k_cache, v_cache, out, T, H, Lmax, d, scale, table, size, range_max, workspace,
                             static_cast<cudaStream_t>(stream), static_cast<int64_t>(Lmax) * d, lens, len_add);
}

}  // extern "C"
