// Batched token sampling with the exp-LUT softmax on B200 (sm_100a).
//
// Reference: BatchedRolloutCoordinator.sample_tokens, NumPy branch
// (antigravity-engine/src/batch_generator.py:187-253), with safe_softmax_lut
// (attention.py:97-134) on a 32,768-entry table over [-10, 0]:
//   greedy (T <= 0) : token = first index of the largest logit; logprob =
//                     fp16(log(p_token)), p = the fp16 LUT softmax of the raw logits;
//   T > 0           : s = logits / max(T, 1e-5) (fp16 logits: fp16 quotient of the fp32
//                     values by fp16(T); fp32 logits: fp32 quotient), p = fp16 LUT
//                     softmax of s, the top-k (k = min(50, V)) of p renormalised, one
//                     draw; logprob = log(max(p_token, 1e-10)) in fp32.
// Defined where the reference leaves it open: the row sum of the fp16 table values is
// exact (integer units of 2^-24) and rounded to fp32 once; the top-k set and its order
// are by (p descending, column ascending); the draw takes the first candidate whose
// running fp32 sum exceeds u * total for a uniform u in [0, 1) (given, or the
// counter-based SplitMix64 stream below). A row whose (scaled) maximum is not finite
// makes the reference raise; here it sets MB_DEVERR_NONFINITE, token = the argmax,
// logprob = NaN.
//
// One cluster of C <= 8 CTAs (1024 threads each) per row, CTA r owning a contiguous
// column range; row-wide sums, maxima and histograms are joined through distributed
// shared memory:
//   A  max and first argmax of the raw logits (the scaled maximum is the scaled value
//      at that column: the scaling is monotone);
//   B  per element the table index of (s - max) into a uint16 scratch row, and the
//      exact sum of the table values (uint64);
//   p16 table: for every table index its fp16 probability fp16(e / sum), in shared
//      memory (the probability of an element is a function of its index alone);
//   C, D  256-bin histograms of the high, then the low byte of the fp16 probability
//      bits give the k-th largest probability t;
//   E  every column with p > t, and the first (k - #{p > t}) columns with p == t in
//      column order (per-thread contiguous ranges, a block prefix sum, and the tie
//      counts of the lower-ranked CTAs);
//   the leader CTA gathers the <= 64 candidate keys (p << 32 | ~column), a warp ranks
//   them, thread 0 draws.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace mb {

constexpr int kSampBlock = 1024;
constexpr int kSampMaxK = 64;

__device__ __forceinline__ int samp_lut_index(float x, float step, int size) {
  float f = __fdiv_rn(fabsf(x), step);
  f = fminf(fmaxf(f, 0.0f), static_cast<float>(size - 1));
  return static_cast<int>(f);
}

struct SampArgs {
  const void* logits;
  int f32;  // 1: fp32 logits, 0: fp16
  int V;
  int scale;    // 0: greedy (raw logits)
  float tdiv;   // fp32(max(T, 1e-5)), or its fp16 rounding for fp16 logits
  int k;
  const uint16_t* table;
  int size;
  float step;
  const float* uniforms;  // [N] or null
  unsigned long long seed;
  uint32_t* rng_state;  // {counter, arrivals}
  int32_t* tokens;
  float* logprobs;
  uint16_t* scratch;  // [N][V] table indices
  uint32_t* err;
};

__device__ __forceinline__ float samp_raw(const SampArgs& a, int64_t i) {
  return a.f32 ? __ldg(static_cast<const float*>(a.logits) + i)
               : __half2float(__ushort_as_half(__ldg(static_cast<const uint16_t*>(a.logits) + i)));
}

__device__ __forceinline__ float samp_scaled(const SampArgs& a, float x) {
  if (!a.scale) return x;
  const float q = __fdiv_rn(x, a.tdiv);
  return a.f32 ? q : __half2float(__float2half_rn(q));
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Block reductions (1024 threads = 32 warps); `red` holds 32 slots.
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long t = 0;
#pragma unroll
  for (int w = 0; w < kSampBlock / 32; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x > v ? x : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long t = 0;
#pragma unroll
  for (int w = 0; w < kSampBlock / 32; ++w) t = red[w] > t ? red[w] : t;
  return t;
}

// Order-preserving 32-bit code of an fp32 value for the argmax: NaN largest, -0 == +0.
__device__ __forceinline__ uint32_t samp_code(float v) {
  if (v != v) return 0xFFFFFFFFu;
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// The bin holding the `need`-th largest element, walking the 256 bins from the top, by
// one warp: lane l sums bins 255-8l .. 248-8l, a scan over the lanes
// (highest bins first) finds the lane holding the `need`-th largest element, which walks
// its 8 bins. All 32 lanes call it; every lane returns the bin and `above` (the count
// of elements in higher bins).
__device__ __forceinline__ int pick_bin_warp(const uint32_t* hist, uint32_t need, uint32_t* above) {
  const int lane = threadIdx.x & 31;
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += hist[255 - 8 * lane - i];
  uint32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  const unsigned hit = __ballot_sync(0xffffffffu, incl >= need);
  const int f = hit ? __ffs(hit) - 1 : 31;
  int bin = 0;
  uint32_t ab = 0;
  if (lane == f) {
    uint32_t cum = incl - s;
    bin = 255 - 8 * lane - 7;
    ab = cum;
    for (int i = 0; i < 8; ++i) {
      const int b = 255 - 8 * lane - i;
      if (cum + hist[b] >= need) {
        bin = b;
        ab = cum;
        break;
      }
      cum += hist[b];
    }
  }
  bin = __shfl_sync(0xffffffffu, bin, f);
  *above = __shfl_sync(0xffffffffu, ab, f);
  return bin;
}

__device__ __forceinline__ unsigned long long ld_cluster_u64(const void* local, uint32_t rank) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(mapa_shared(smem_u32(local), rank)) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_cluster_u32(const void* local, uint32_t rank) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(mapa_shared(smem_u32(local), rank)) : "memory");
  return v;
}

// One cluster of gridDim.x CTAs per row (blockIdx.y); CTA r of the cluster owns the
// contiguous columns [r * chunk, (r + 1) * chunk). Row-wide values are reduced through
// distributed shared memory: each CTA publishes its partial in its own shared memory,
// a cluster barrier, then every CTA (or the leader, rank 0) reads the partials of all
// ranks in rank order. Every CTA of a cluster takes the same branches (they derive
// from row-wide values), so all pass the same cluster barriers.
__global__ void __launch_bounds__(kSampBlock, 1) k_sample(SampArgs a) {
  extern __shared__ uint16_t ptab[];  // [size] fp16 probability bits per table index
  __shared__ unsigned long long red[kSampBlock / 32];
  __shared__ unsigned long long part_a, part_b, bcast;
  __shared__ uint32_t hist_c[256], hist_d[256], gh[256];
  __shared__ uint32_t scan[kSampBlock / 32];
  __shared__ unsigned long long lc[kSampMaxK], lt[kSampMaxK], cand[kSampMaxK], sorted[kSampMaxK];
  __shared__ uint32_t lcn, ltn, lties;
  __shared__ uint32_t gcnt[2 * 8 + 1];  // leader: per-rank candidate counts (> t, then ties) and their prefix
  __shared__ uint32_t sel[4];  // bin, above, threshold, c_gt
  // the exp table into shared memory (it does not depend on the previous kernel, so
  // this overlaps its tail); ptab holds table[j] until it becomes the probability table
  if ((a.size & 7) == 0 && (reinterpret_cast<uintptr_t>(a.table) & 15) == 0) {
    for (int j = threadIdx.x; j < a.size / 8; j += kSampBlock)
      reinterpret_cast<uint4*>(ptab)[j] = __ldg(reinterpret_cast<const uint4*>(a.table) + j);
  } else {
    for (int j = threadIdx.x; j < a.size; j += kSampBlock) ptab[j] = __ldg(a.table + j);
  }
  pdl_wait();
  pdl_launch_dependents();
  const int C = static_cast<int>(gridDim.x);
  const uint32_t r = cluster_ctarank();
  const int n = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t row = static_cast<int64_t>(n) * a.V;
  uint16_t* srow = a.scratch + row;
  const int chunk = (a.V + C - 1) / C;
  const int cb = min(a.V, static_cast<int>(r) * chunk), ce = min(a.V, cb + chunk);
  if (tid == 0) {
    lcn = 0;
    ltn = 0;
    lties = 0;
  }
  for (int b = tid; b < 256; b += kSampBlock) {
    hist_c[b] = 0;
    hist_d[b] = 0;
  }

  // A: first index of the largest raw logit (NaN largest), row-wide
  constexpr int kU = 8;  // loads issued before any is used
  unsigned long long best = 0;
  for (int base = cb + tid; base < ce; base += kU * kSampBlock) {
    float v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + u * kSampBlock;
      v[u] = c < ce ? samp_raw(a, row + c) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + u * kSampBlock;
      const unsigned long long key =
          (static_cast<unsigned long long>(samp_code(v[u])) << 32) | (0xFFFFFFFFull - c);
      if (c < ce) best = key > best ? key : best;
    }
  }
  best = block_max_u64(best, red);  // its barriers also publish the staged table
  if (tid == 0) part_a = best;
  cluster_sync();
  if (tid == 0) {
    unsigned long long b = 0;
    for (int q = 0; q < C; ++q) {
      const unsigned long long v = ld_cluster_u64(&part_a, q);
      b = v > b ? v : b;
    }
    bcast = b;
  }
  __syncthreads();
  best = bcast;
  const int amax = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  const float m = samp_scaled(a, samp_raw(a, row + amax));
  const uint32_t counter = *reinterpret_cast<volatile uint32_t*>(a.rng_state);
  const bool leader = r == 0;
  if (!isfinite(m)) {  // the reference raises on a non-finite maximum
    if (leader && tid == 0) {
      if (a.err) atomicOr(a.err, MB_DEVERR_NONFINITE);
      a.tokens[n] = amax;
      a.logprobs[n] = __int_as_float(0x7fc00000);
    }
  } else {
    // B: table indices and the exact sum of the table values, row-wide
    unsigned long long acc = 0;
    for (int base = cb + tid; base < ce; base += kU * kSampBlock) {
      float v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = base + u * kSampBlock;
        v[u] = c < ce ? samp_raw(a, row + c) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = base + u * kSampBlock;
        if (c < ce) {
          const int j = samp_lut_index(samp_scaled(a, v[u]) - m, a.step, a.size);
          if (a.scale) srow[c] = static_cast<uint16_t>(j);
          const float e = __half2float(__ushort_as_half(ptab[a.size - 1 - j]));
          acc += static_cast<unsigned long long>(e * 16777216.0f);  // exact: e is a multiple of 2^-24, <= 1
        }
      }
    }
    acc = block_sum_u64(acc, red);
    if (tid == 0) part_b = acc;
    cluster_sync();
    if (tid == 0) {
      unsigned long long t = 0;
      for (int q = 0; q < C; ++q) t += ld_cluster_u64(&part_b, q);
      bcast = t;
    }
    __syncthreads();
    float sum = __ull2float_rn(bcast) * 5.9604644775390625e-8f;  // * 2^-24, exact
    if (!(sum > 0.0f)) sum = 1.0f;
    if (!a.scale) {
      if (leader && tid == 0) {
        const float e0 = __half2float(__ushort_as_half(ptab[a.size - 1]));
        const float p = __half2float(__float2half_rn(__fdiv_rn(e0, sum)));
        a.tokens[n] = amax;
        a.logprobs[n] = __half2float(__float2half_rn(logf(p)));
      }
    } else {
      // probability bits per table index, in place: ptab[j] = fp16(table[S-1-j] / sum)
      // (entries j and S-1-j swap, one thread per pair)
      for (int j = tid; j < (a.size + 1) / 2; j += kSampBlock) {
        const int jj = a.size - 1 - j;
        const float lo = __half2float(__ushort_as_half(ptab[j])), hi = __half2float(__ushort_as_half(ptab[jj]));
        ptab[j] = __half_as_ushort(__float2half_rn(__fdiv_rn(hi, sum)));
        ptab[jj] = __half_as_ushort(__float2half_rn(__fdiv_rn(lo, sum)));
      }
      __syncthreads();
      const uint32_t k = static_cast<uint32_t>(a.k);
      // C: high byte histogram, row-wide
      for (int base = cb; base < ce; base += kU * kSampBlock) {  // trip count uniform over the warp
        uint32_t jv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = base + u * kSampBlock + tid;
          jv[u] = c < ce ? __ldcg(srow + c) : 0xFFFFu;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int bin = jv[u] != 0xFFFFu ? (ptab[jv[u]] >> 8) : -1;
          const unsigned peers = __match_any_sync(0xffffffffu, bin);
          if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist_c[bin], static_cast<uint32_t>(__popc(peers)));
        }
      }
      __syncthreads();
      cluster_sync();
      if (tid < 256) {
        uint32_t t = 0;
        for (int q = 0; q < C; ++q) t += ld_cluster_u32(&hist_c[tid], q);
        gh[tid] = t;
      }
      __syncthreads();
      if (tid < 32) {
        uint32_t above;
        const int b = pick_bin_warp(gh, k, &above);
        if (tid == 0) {
          sel[0] = static_cast<uint32_t>(b);
          sel[1] = above;
        }
      }
      __syncthreads();
      const uint32_t hb = sel[0], above_hi = sel[1];
      // D: low byte histogram inside the high bin, row-wide
      for (int base = cb; base < ce; base += kU * kSampBlock) {
        uint32_t jv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = base + u * kSampBlock + tid;
          jv[u] = c < ce ? __ldcg(srow + c) : 0xFFFFu;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          int bin = -1;
          if (jv[u] != 0xFFFFu) {
            const uint32_t p = ptab[jv[u]];
            if ((p >> 8) == hb) bin = static_cast<int>(p & 0xFFu);
          }
          const unsigned peers = __match_any_sync(0xffffffffu, bin);
          if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist_d[bin], static_cast<uint32_t>(__popc(peers)));
        }
      }
      __syncthreads();
      cluster_sync();
      if (tid < 256) {
        uint32_t t = 0;
        for (int q = 0; q < C; ++q) t += ld_cluster_u32(&hist_d[tid], q);
        gh[tid] = t;
      }
      __syncthreads();
      if (tid < 32) {
        uint32_t above;
        const int lo = pick_bin_warp(gh, k - above_hi, &above);
        if (tid == 0) {
          sel[2] = (hb << 8) | static_cast<uint32_t>(lo);
          sel[3] = above_hi + above;
        }
      }
      __syncthreads();
      const uint32_t t = sel[2], c_gt = sel[3];
      const uint32_t need = k - c_gt;  // >= 1 columns with p == t, the first ones by column
      // E: contiguous column range per thread inside this CTA's range, in column order
      const int sub = (ce - cb + kSampBlock - 1) / kSampBlock;
      const int c0 = min(ce, cb + tid * sub), c1 = min(ce, c0 + sub);
      uint32_t ties = 0;
      for (int cc = c0; cc < c1; cc += kU) {
        uint32_t jv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) jv[u] = cc + u < c1 ? __ldcg(srow + cc + u) : 0u;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = cc + u;
          if (c >= c1) break;
          const uint32_t p = ptab[jv[u]];
          if (p > t) {
            const uint32_t slot = atomicAdd(&lcn, 1u);
            if (slot < kSampMaxK) lc[slot] = (static_cast<unsigned long long>(p) << 32) | (0xFFFFFFFFull - c);
          } else if (p == t) {
            ++ties;
          }
        }
      }
      // exclusive prefix of the tie counts over threads (thread order = column order)
      uint32_t incl = ties;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      if (lane == 31) scan[tid >> 5] = incl;
      __syncthreads();
      if (tid < 32) {
        const uint32_t v = scan[tid];
        uint32_t s2 = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t x = __shfl_up_sync(0xffffffffu, s2, o);
          if (lane >= o) s2 += x;
        }
        scan[tid] = s2 - v;  // exclusive over warps
        if (tid == 31) lties = s2;  // this CTA's tie count
      }
      __syncthreads();
      cluster_sync();  // tie counts of every rank published
      if (tid == 0) {
        uint32_t off = 0;
        for (uint32_t q = 0; q < r; ++q) off += ld_cluster_u32(&lties, q);
        sel[0] = off;  // ties in lower ranks' columns
        ltn = off >= need ? 0u : min(lties, need - off);
      }
      __syncthreads();
      const uint32_t lim = ltn;
      uint32_t rank = scan[tid >> 5] + incl - ties;  // local rank among this CTA's ties
      for (int cc = c0; cc < c1 && ties > 0 && rank < lim; cc += kU) {
        uint32_t jv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) jv[u] = cc + u < c1 ? __ldcg(srow + cc + u) : 0u;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = cc + u;
          if (c < c1 && rank < lim && ptab[jv[u]] == t) {
            lt[rank] = (static_cast<unsigned long long>(t) << 32) | (0xFFFFFFFFull - c);
            ++rank;
          }
        }
      }
      __syncthreads();
      cluster_sync();  // candidate lists of every rank published
      if (leader) {
        // gather the ranks' lists: counts first (one thread per list), then one
        // thread per candidate, so the remote loads overlap
        if (tid < 2 * C) {
          const int q = tid % C;
          gcnt[tid] = tid < C ? min(ld_cluster_u32(&lcn, q), static_cast<uint32_t>(kSampMaxK))
                              : ld_cluster_u32(&ltn, q);
        }
        __syncthreads();
        if (tid < static_cast<int>(k)) {
          uint32_t i = static_cast<uint32_t>(tid), list = 0;
          while (list < static_cast<uint32_t>(2 * C) && i >= gcnt[list]) i -= gcnt[list++];
          unsigned long long key = 0;  // unreachable zero when the counts agree
          if (list < static_cast<uint32_t>(2 * C)) {
            const uint32_t q = list % C;
            key = list < static_cast<uint32_t>(C) ? ld_cluster_u64(&lc[i], q) : ld_cluster_u64(&lt[i], q);
          }
          cand[tid] = key;
        }
        __syncthreads();
        // rank the k candidate keys (distinct: the column is part of the key)
        if (tid < 32) {
          for (uint32_t i = tid; i < k; i += 32) {
            const unsigned long long key = cand[i];
            uint32_t rk = 0;
            for (uint32_t j = 0; j < k; ++j) rk += cand[j] > key ? 1u : 0u;
            sorted[rk] = key;
          }
        }
        __syncthreads();
        if (tid == 0) {
          float u;
          if (a.uniforms) {
            u = a.uniforms[n];
          } else {
            const unsigned long long base =
                splitmix64(a.seed ^ (static_cast<unsigned long long>(counter) * 0xD1B54A32D192ED03ull));
            u = static_cast<float>(splitmix64(base + static_cast<unsigned long long>(n)) >> 40) *
                5.9604644775390625e-8f;
          }
          float total = 0.0f;
          for (uint32_t i = 0; i < k; ++i)
            total += __half2float(__ushort_as_half(static_cast<uint16_t>(sorted[i] >> 32)));
          uint32_t pick = k - 1;
          if (total > 0.0f) {
            const float target = u * total;
            float run = 0.0f;
            for (uint32_t i = 0; i < k; ++i) {
              run += __half2float(__ushort_as_half(static_cast<uint16_t>(sorted[i] >> 32)));
              if (run > target) {
                pick = i;
                break;
              }
            }
          } else {
            pick = min(static_cast<uint32_t>(floorf(u * static_cast<float>(k))), k - 1);
          }
          const unsigned long long key = sorted[pick];
          const float p = __half2float(__ushort_as_half(static_cast<uint16_t>(key >> 32)));
          a.tokens[n] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
          a.logprobs[n] = logf(fmaxf(p, 1e-10f));
        }
      }
    }
  }
  // no CTA leaves while the leader may still read its shared memory
  cluster_sync();
  // the last row's leader advances the random stream's counter (read by the next call)
  if (leader && tid == 0) {
    __threadfence();
    if (atomicAdd(a.rng_state + 1, 1u) == gridDim.y - 1) {
      a.rng_state[1] = 0;
      a.rng_state[0] = counter + 1;
      __threadfence();
    }
  }
}

}  // namespace mb

using namespace mb;

// Per device, once: the kernel's shared-memory limit and how many clusters of each
// size (1 CTA of 1024 threads and 64 KB + static shared memory per SM) fit at once.
constexpr int kSampMaxDevices = 64;
struct SampDevice {
  bool ready = false;
  int capacity[9] = {};
};
static SampDevice g_samp_dev[kSampMaxDevices];
static std::once_flag g_samp_once[kSampMaxDevices];

static SampDevice& samp_device(int dev) {
  std::call_once(g_samp_once[dev], [dev] {
    SampDevice& sd = g_samp_dev[dev];
    const int smem = 32768 * static_cast<int>(sizeof(uint16_t));
    if (cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sd.capacity[1] = sms;
    for (int c = 2; c <= 8; ++c) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, 1);
      cfg.blockDim = dim3(kSampBlock);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = c;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_sample, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
      }
      sd.capacity[c] = n;
    }
    sd.ready = true;
  });
  return g_samp_dev[dev];
}

extern "C" {

size_t mb_sample_workspace_size(int32_t N, int32_t V) {
  if (N < 1 || V < 1) return 0;
  return (static_cast<size_t>(N) * V * sizeof(uint16_t) + 255) / 256 * 256;
}

int32_t mb_sample_tokens(const void* logits, int32_t logits_f32, int32_t N, int32_t V, float temperature,
                         int32_t top_k, const uint16_t* table, int32_t size, float range_max, const float* uniforms,
                         uint64_t seed, uint32_t* rng_state, int32_t* tokens, float* logprobs, void* workspace,
                         size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  if (!logits || !table || !rng_state || !tokens || !logprobs || !workspace) return MB_ERR_NULL;
  if (N < 1 || V < 1 || V > 0x7FFFFFFE || size < 2 || size > 32768 || !(range_max > 0.0f) || top_k < 1 ||
      top_k > kSampMaxK || (logits_f32 != 0 && logits_f32 != 1))
    return MB_ERR_ARGS;
  if (workspace_bytes < mb_sample_workspace_size(N, V)) return MB_ERR_WORKSPACE;
  SampArgs a;
  a.logits = logits;
  a.f32 = logits_f32;
  a.V = V;
  a.scale = temperature > 0.0f ? 1 : 0;
  const float t32 = fmaxf(temperature, 1e-5f);
  a.tdiv = logits_f32 ? t32 : __half2float(__float2half_rn(t32));
  a.k = top_k < V ? top_k : V;
  a.table = table;
  a.size = size;
  a.step = static_cast<float>(static_cast<double>(range_max) / (size - 1));
  a.uniforms = uniforms;
  a.seed = seed;
  a.rng_state = rng_state;
  a.tokens = tokens;
  a.logprobs = logprobs;
  a.scratch = static_cast<uint16_t*>(workspace);
  a.err = dev_err;
  const size_t smem = static_cast<size_t>(size) * sizeof(uint16_t);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kSampMaxDevices) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  SampDevice& sd = samp_device(dev);
  if (!sd.ready) return MB_ERR_LAUNCH;
  // cluster size: the largest C <= 8 whose N clusters are resident at once (one wave)
  int C = 1;
  for (int c = 8; c >= 2; --c)
    if (sd.capacity[c] >= N) {
      C = c;
      break;
    }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, N);
  cfg.blockDim = dim3(kSampBlock);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, k_sample, a) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return launch_status();
}

}  // extern "C"
