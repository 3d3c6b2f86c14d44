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
// One cluster of C <= 16 CTAs (1024 threads each) per row, CTA r owning a contiguous
// column range of a multiple of 8 columns (8-column groups, one 16-byte load each when
// the rows are aligned), and a 16-bit column buffer of table indices per CTA in shared
// memory (in the global scratch row when it does not fit). Three row-wide joins, each
// a push of partials into the other CTAs' shared memory (distributed shared memory)
// and one cluster barrier:
//   A  max and first argmax of the raw logits, on order-preserving integer codes (the
//      scaled maximum is the scaled value at that column: the scaling is monotone);
//   B  per column the table index j of (s - max): the index is a non-increasing
//      function of the column's code, so a per-CTA table of the highest codes below the
//      maximum gives it by one lookup, and every code below a table whose lowest entry
//      clips (most of a row) gets the clip index size - 1 by one compare; j goes to the
//      column buffer, the exact sum of the table values is joined (uint64 units of
//      2^-24);
//   C..E  the probability p(j) = fp16(table[S-1-j] / sum) is a non-increasing function
//      of j, and the row's top-k by (p descending, column ascending) lies in the union
//      of the CTAs' own top-k: each CTA finds its k-th smallest index j_k (T > 0 on
//      aligned fp16 rows: pass B counted the unclipped columns per code-table offset,
//      and j_k follows from a block prefix over the counts; otherwise a high-bit
//      histogram, then one of the low 7 bits inside the chosen bin), the indices
//      [j_lo, j_hi] whose probability equals p(j_k) (two warps, 32-way searches of p,
//      first over the 32 indices next to j_k),
//      and takes every column below j_lo and the first ties in column order (a block
//      prefix sum); it sorts these keys (p << 32 | ~column) and pushes them to the
//      leader CTA, which ranks every key of the union by binary searches in the
//      other lists, and thread 0 draws.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace mb {

constexpr int kSampBlock = 1024;
constexpr int kSampMaxK = 64;
constexpr int kSampMaxCluster = 16;  // CTAs per row (sizes above 8 are non-portable)
constexpr int kSampLd = 1;           // 8-column groups whose loads a thread issues together
constexpr int kSampLutMax = 4096;    // codes below the maximum in the code -> index table

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
  float clip;  // |s - max| >= clip implies table index size - 1 (no division needed)
  const float* uniforms;  // [N] or null
  unsigned long long seed;
  uint32_t* rng_state;  // {counter, arrivals}
  int32_t* tokens;
  float* logprobs;
  uint16_t* scratch;  // [N][V] column buffers when a CTA's columns do not fit shared memory
  int chunk;          // columns per CTA of a cluster (a multiple of 8)
  int buf_smem;       // 1: the column buffer lives in shared memory after the table
  int lut_off;        // code -> index table: offset (uint16 entries) in dynamic shared memory
  int lut_cap;        // and capacity (entries)
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

// Block reductions (1024 threads = 32 warps) whose result only warp 0 needs (it pushes
// the CTA's partial to the cluster): the warps' partials meet in `red` (32 slots), and
// warp 0 reduces them with shuffles. Both barriers also order every earlier
// shared-memory write of the block before whatever warp 0 does next.
__device__ __forceinline__ unsigned long long block_sum_u64_w0(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  return v;
}

__device__ __forceinline__ unsigned long long block_max_u64_w0(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x > v ? x : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
      v = x > v ? x : v;
    }
  }
  return v;
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

// Order-preserving 32-bit codes of logits (NaN largest, -0 == +0) and their inverses
// for non-NaN codes: fp16 bit patterns, fp32 values.
__device__ __forceinline__ uint32_t code16(uint32_t h) {
  if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu) != 0u) return 0xFFFFu;
  if (h == 0x8000u) h = 0u;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
__device__ __forceinline__ float decode16(uint32_t c) {
  const uint32_t h = (c & 0x8000u) ? (c & 0x7FFFu) : (~c & 0xFFFFu);
  return __half2float(__ushort_as_half(static_cast<uint16_t>(h)));
}
__device__ __forceinline__ float decode32(uint32_t c) { return __uint_as_float((c & 0x80000000u) ? (c & 0x7FFFFFFFu) : ~c); }

// Codes of the eight columns [c, c + 8) (VEC: one or two 16-byte loads); columns at or
// past `ce` get code 0, below every value.
template <bool VEC>
__device__ __forceinline__ void samp_codes8(const SampArgs& a, int64_t row, int c, int ce, uint32_t (&k)[8]) {
  if (a.f32) {
    float v[8];
    if (VEC && c + 8 <= ce) {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.logits) + row + c);
      const float4 x = __ldg(p), y = __ldg(p + 1);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
      v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = c + u < ce ? __ldg(static_cast<const float*>(a.logits) + row + c + u) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) k[u] = c + u < ce ? samp_code(v[u]) : 0u;
  } else {
    uint32_t h[8];
    if (VEC && c + 8 <= ce) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.logits) + row + c));
      h[0] = q.x & 0xFFFFu; h[1] = q.x >> 16; h[2] = q.y & 0xFFFFu; h[3] = q.y >> 16;
      h[4] = q.z & 0xFFFFu; h[5] = q.z >> 16; h[6] = q.w & 0xFFFFu; h[7] = q.w >> 16;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) h[u] = c + u < ce ? __ldg(static_cast<const uint16_t*>(a.logits) + row + c + u) : 0u;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) k[u] = c + u < ce ? code16(h[u]) : 0u;
  }
}

__device__ __forceinline__ void st_cluster_u32(const void* local, uint32_t rank, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(smem_u32(local), rank)), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u64(const void* local, uint32_t rank, unsigned long long v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(mapa_shared(smem_u32(local), rank)), "l"(v) : "memory");
}

// First code in [lo, hi] at which the monotone predicate (true, ..., true, false, ...)
// is false, given pred(hi) == false; 32 probes per round by one warp.
template <typename Pred>
__device__ __forceinline__ uint32_t warp_first_false(uint32_t lo, uint32_t hi, Pred pred) {
  const int lane = threadIdx.x & 31;
  while (lo < hi) {
    const uint32_t stp = (hi - lo) / 31u + 1u;  // 31 steps reach past hi: lane 31 probes hi
    const uint32_t c = min(hi, lo + static_cast<uint32_t>(lane) * stp);
    const unsigned bal = __ballot_sync(0xffffffffu, !pred(c));
    const int f = __ffs(bal) - 1;
    const uint32_t cf = min(hi, lo + static_cast<uint32_t>(f) * stp);
    if (f > 0) lo = min(hi, lo + static_cast<uint32_t>(f - 1) * stp) + 1u;
    hi = cf;
  }
  return lo;
}

// The same order-preserving code for the fast path, two fp16 columns per 32-bit word
// (negative: ~h, else h | 0x8000; -0 and +0 get neighbouring codes, which order and
// decode the same way; NaNs are detected separately).
__device__ __forceinline__ uint32_t code16p(uint32_t h) { return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u); }
__device__ __forceinline__ uint32_t code16x2(uint32_t w) {
  const uint32_t m = ((w & 0x80008000u) >> 15) * 0xFFFFu;  // 0xFFFF in each negative half
  return (w ^ m) | (0x80008000u & ~m);
}

template <bool VEC>
__device__ __forceinline__ void buf_load8(const uint16_t* buf, int o, int n, uint32_t (&w)[8]) {
  if (VEC && o + 8 <= n) {
    const uint4 q = *reinterpret_cast<const uint4*>(buf + o);
    w[0] = q.x & 0xFFFFu; w[1] = q.x >> 16; w[2] = q.y & 0xFFFFu; w[3] = q.y >> 16;
    w[4] = q.z & 0xFFFFu; w[5] = q.z >> 16; w[6] = q.w & 0xFFFFu; w[7] = q.w >> 16;
  } else {
#pragma unroll
    for (int u = 0; u < 8; ++u) w[u] = o + u < n ? buf[o + u] : 0xFFFFu;
  }
}

template <bool VEC>
__device__ __forceinline__ void buf_store8(uint16_t* buf, int o, int n, const uint32_t (&w)[8]) {
  if (VEC && o + 8 <= n) {
    *reinterpret_cast<uint4*>(buf + o) =
        make_uint4(w[0] | (w[1] << 16), w[2] | (w[3] << 16), w[4] | (w[5] << 16), w[6] | (w[7] << 16));
  } else {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (o + u < n) buf[o + u] = static_cast<uint16_t>(w[u]);
  }
}

// One cluster of gridDim.x CTAs per row (blockIdx.y); CTA r of the cluster owns the
// contiguous columns [r * chunk, (r + 1) * chunk) (chunk a multiple of 8). Row-wide
// values are joined by pushing: each CTA stores its partial into a slot of every CTA
// of the cluster (distributed shared memory), one cluster barrier, then every CTA
// reduces the slots locally in rank order. Every CTA of a cluster takes the same
// branches (they derive from row-wide values), so all pass the same cluster barriers,
// and no CTA touches another's shared memory after the last barrier it passes.
// Shared memory: the exp table, then the 16-bit column buffer of table indices (in the
// row's global scratch when it does not fit).
template <bool VEC>
__global__ void __launch_bounds__(kSampBlock, 1) k_sample(SampArgs a) {
  extern __shared__ __align__(16) uint16_t ptab[];  // [size] the exp table, then the column buffer
  __shared__ unsigned long long red[kSampBlock / 32];
  __shared__ unsigned long long xa[kSampMaxCluster], xb[kSampMaxCluster];  // pushed: max keys, sums
  __shared__ unsigned long long xa2[kSampMaxCluster];  // pushed: argmax keys of an erring row (fast path)
  __shared__ unsigned long long xlist[kSampMaxCluster][kSampMaxK];  // pushed to the leader: sorted local top-k
  __shared__ uint32_t xlen[kSampMaxCluster];
  __shared__ uint32_t hist[256], hist2[256];  // high-bit, then low-bit histograms of this CTA's indices
  __shared__ uint32_t icnt[kSampLutMax];       // fast path: columns per code-table offset
  __shared__ uint32_t scan[kSampBlock / 32];
  __shared__ unsigned long long lc[kSampMaxK], sorted[kSampMaxK];
  __shared__ unsigned long long bcast;
  __shared__ uint32_t lcn, lties;
  __shared__ uint32_t sel[4];  // histogram picks, then j_lo, j_hi and the fp16 bits of p(j_k)
  // the exp table into shared memory (it does not depend on the previous kernel, so
  // this overlaps its tail)
  if ((a.size & 7) == 0 && (reinterpret_cast<uintptr_t>(a.table) & 15) == 0) {
    for (int j = threadIdx.x; j < a.size / 8; j += kSampBlock)
      reinterpret_cast<uint4*>(ptab)[j] = __ldg(reinterpret_cast<const uint4*>(a.table) + j);
  } else {
    for (int j = threadIdx.x; j < a.size; j += kSampBlock) ptab[j] = __ldg(a.table + j);
  }
  if (threadIdx.x == 0) {
    lcn = 0;
    lties = 0;
  }
  for (int b = threadIdx.x; b < 256; b += kSampBlock) {
    hist[b] = 0;
    hist2[b] = 0;
  }
  for (int b = threadIdx.x; b < kSampLutMax; b += kSampBlock) icnt[b] = 0;
  cluster_arrive_relaxed();  // phase 0: this CTA runs (awaited before the first remote store)
  pdl_wait();
  pdl_launch_dependents();
  const int C = static_cast<int>(gridDim.x);
  const uint32_t r = cluster_ctarank();
  const int n = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t row = static_cast<int64_t>(n) * a.V;
  const int cb = min(a.V, static_cast<int>(r) * a.chunk), ce = min(a.V, cb + a.chunk);
  const int nc = ce - cb;  // this CTA's columns
  uint16_t* buf = a.buf_smem ? ptab + ((a.size + 7) & ~7) : a.scratch + row + cb;

  // A: first index of the largest raw logit (NaN largest), row-wide, on the codes. The
  // common case (T > 0, fp16 rows on 16-byte boundaries) needs only the maximum value:
  // two columns per packed max; the column is found later only if the row errs.
  const bool fast = VEC && a.scale && !a.f32;
  uint32_t bcode = 0;
  int bcol = -1;
  if (fast) {
    uint32_t vmx = 0, nanm = 0;
    const uint16_t* xr = static_cast<const uint16_t*>(a.logits) + row + cb;
    for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
      if (o + 8 <= nc) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + o));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          vmx = __vmaxu2(vmx, code16x2(w[i]));
          nanm |= __vcmpgtu2(w[i] & 0x7FFF7FFFu, 0x7C007C00u);
        }
      } else {
        for (int u = 0; o + u < nc; ++u) {
          const uint32_t h = __ldg(xr + o + u);
          vmx = __vmaxu2(vmx, code16p(h));
          nanm |= (h & 0x7FFFu) > 0x7C00u ? 1u : 0u;
        }
      }
    }
    bcode = nanm ? 0xFFFFu : max(vmx & 0xFFFFu, vmx >> 16);
  } else {
    for (int o = tid * 8; o < nc; o += kSampLd * 8 * kSampBlock) {  // kSampLd groups' loads in flight
      uint32_t k8[kSampLd][8];
#pragma unroll
      for (int g = 0; g < kSampLd; ++g) samp_codes8<VEC>(a, row, cb + o + g * 8 * kSampBlock, ce, k8[g]);
#pragma unroll
      for (int g = 0; g < kSampLd; ++g)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int oo = o + g * 8 * kSampBlock + u;
          if (oo < nc && (bcol < 0 || k8[g][u] > bcode)) {  // columns ascend: strict > keeps the first
            bcode = k8[g][u];
            bcol = cb + oo;
          }
        }
    }
  }
  unsigned long long best =
      fast ? static_cast<unsigned long long>(bcode) << 32
           : (bcol < 0 ? 0ull
                       : (static_cast<unsigned long long>(bcode) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(bcol)));
  best = block_max_u64_w0(best, red);  // its barriers also publish the staged table
  cluster_wait();                   // phase 0: every CTA of the cluster runs
  if (tid < C) st_cluster_u64(&xa[r], tid, best);
  cluster_sync();
  if (tid < 32) {
    unsigned long long v = lane < C ? xa[lane] : 0ull;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
      v = x > v ? x : v;
    }
    if (tid == 0) bcast = v;
  }
  __syncthreads();
  best = bcast;
  int amax = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  const uint32_t acode = static_cast<uint32_t>(best >> 32);
  const float m = fast ? samp_scaled(a, decode16(acode)) : samp_scaled(a, samp_raw(a, row + amax));
  const uint32_t counter = *reinterpret_cast<volatile uint32_t*>(a.rng_state);
  const bool leader = r == 0;
  if (!isfinite(m)) {  // the reference raises on a non-finite maximum
    if (fast) {  // the erring row's token is the first column of its maximum: one more join
      uint32_t bc = 0;
      int bj = -1;
      for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
        uint32_t k8[8];
        samp_codes8<VEC>(a, row, cb + o, ce, k8);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (o + u < nc && (bj < 0 || k8[u] > bc)) {
            bc = k8[u];
            bj = cb + o + u;
          }
      }
      unsigned long long key =
          bj < 0 ? 0ull : (static_cast<unsigned long long>(bc) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(bj));
      key = block_max_u64_w0(key, red);
      if (tid < C) st_cluster_u64(&xa2[r], tid, key);
      cluster_sync();
      if (tid < 32) {
        unsigned long long v = lane < C ? xa2[lane] : 0ull;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
          v = x > v ? x : v;
        }
        if (tid == 0) bcast = v;
      }
      __syncthreads();
      amax = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(bcast & 0xFFFFFFFFull));
    }
    if (leader && tid == 0) {
      if (a.err) atomicOr(a.err, MB_DEVERR_NONFINITE);
      a.tokens[n] = amax;
      a.logprobs[n] = __int_as_float(0x7fc00000);
    }
  } else {
    const int jclip = a.size - 1;
    // Code -> index table for the highest codes up to the maximum (fp16 logits): j of a
    // column is a non-increasing function of its code, so once the table's lowest code
    // clips, every code below it clips too, and a column costs one compare or one
    // lookup instead of two divisions. Codes below a table that does not reach the clip
    // index (a flat row) take the exact path.
    // The table grows downwards from the maximum in slices of one code per thread, and
    // stops at the first slice whose lowest code clips (one slice for most rows).
    const uint32_t lo_code = a.f32 ? 0x007FFFFFu : 0x03FFu;  // code of -inf
    const uint32_t lmax = a.f32 ? 0u : min(acode - lo_code + 1u, static_cast<uint32_t>(min(a.lut_cap, kSampLutMax)));
    uint16_t* cj = ptab + a.lut_off;  // cj[i]: index of code acode - i
    uint32_t lw = 0;
    bool below_clip = false;
    while (lw < lmax && !below_clip) {  // CTA-uniform
      const uint32_t i = lw + tid;
      if (i < lmax) cj[i] = static_cast<uint16_t>(samp_lut_index(samp_scaled(a, decode16(acode - i)) - m, a.step, a.size));
      lw = min(lmax, lw + kSampBlock);
      __syncthreads();
      below_clip = cj[lw - 1] == static_cast<uint16_t>(jclip);
    }
    const uint32_t lut_lo = acode + 1u - lw;  // lowest code of the table
    // B: table indices and the exact sum of the table values (in units of 2^-24: every
    // table value is a multiple of 2^-24, <= 1). With T > 0 the indices go to the column
    // buffer, and the high bits of those below the clip index into this CTA's
    // histogram, bin 255 - (j >> 7) (the bins of the smallest indices, the largest
    // probabilities, come first).
    unsigned long long acc = 0;
    uint32_t nclip = 0;
    // one column whose index is not settled by the group test: look it up or compute it
    auto settle = [&](int o, uint32_t c) {
      int j;
      if (below_clip && c < lut_lo)
        j = jclip;
      else if (lw > 0 && c >= lut_lo)
        j = cj[acode - c];
      else
        j = samp_lut_index(samp_scaled(a, a.f32 ? decode32(c) : decode16(c)) - m, a.step, a.size);
      if (a.scale) buf[o] = static_cast<uint16_t>(j);
      if (j == jclip) {
        ++nclip;
      } else {
        acc += static_cast<uint32_t>(__half2float(__ushort_as_half(ptab[a.size - 1 - j])) * 16777216.0f);
        if (a.scale) atomicAdd(&hist[255 - (j >> 7)], 1u);
      }
    };
    // Fast path with a code table that reaches the clip index: an unclipped column's
    // index is cj[i] of its table offset i = acode - code, a non-decreasing function of
    // i, so pass B only counts the columns per offset (icnt) and leaves i (or 0xFFFF
    // for a clipped column) in the column buffer; the sum, the k-th smallest index and
    // every later classification read the counts and cj.
    const bool fastb = fast && below_clip;
    if (fastb) {
      const uint16_t* xr = static_cast<const uint16_t*>(a.logits) + row + cb;
      const uint32_t lo2 = lut_lo * 0x10001u;
      for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
        if (o + 8 <= nc) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + o));
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
          uint32_t open = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t lt = __vcmpltu2(code16x2(w[i]), lo2);  // 0xFFFF where the column clips
            open |= ((~lt & 1u) | ((~lt >> 15) & 2u)) << (2 * i);
          }
          nclip += 8u - __popc(open);
          *reinterpret_cast<uint4*>(buf + o) = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
          while (open) {
            const int u = __ffs(open) - 1;
            open &= open - 1u;
            const uint32_t word = u < 2 ? w[0] : (u < 4 ? w[1] : (u < 6 ? w[2] : w[3]));
            const uint32_t i = acode - code16p((u & 1) ? (word >> 16) : (word & 0xFFFFu));
            atomicAdd(&icnt[i], 1u);
            buf[o + u] = static_cast<uint16_t>(i);
          }
        } else {
          for (int u = 0; o + u < nc; ++u) {
            const uint32_t c = code16p(__ldg(xr + o + u));
            if (c < lut_lo) {
              buf[o + u] = 0xFFFFu;
              ++nclip;
            } else {
              atomicAdd(&icnt[acode - c], 1u);
              buf[o + u] = static_cast<uint16_t>(acode - c);
            }
          }
        }
      }
      __syncthreads();
      for (uint32_t i = tid; i < lw; i += kSampBlock)
        acc += static_cast<unsigned long long>(icnt[i]) *
               static_cast<uint32_t>(__half2float(__ushort_as_half(ptab[a.size - 1 - cj[i]])) * 16777216.0f);
    } else if (fast) {
      // two columns per packed compare against the table's lowest code; a group whose
      // columns all clip costs one vector store, the others go through `settle` one
      // set bit at a time (a warp pays for its busiest lane, not for every column)
      const uint16_t* xr = static_cast<const uint16_t*>(a.logits) + row + cb;
      const uint32_t lo2 = lut_lo * 0x10001u;
      const uint32_t jj2 = static_cast<uint32_t>(jclip) * 0x10001u;
      for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
        uint32_t w[4] = {0u, 0u, 0u, 0u}, open;
        if (o + 8 <= nc) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + o));
          w[0] = q.x;
          w[1] = q.y;
          w[2] = q.z;
          w[3] = q.w;
          open = 0xFFu;
          if (below_clip) {
            open = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t lt = __vcmpltu2(code16x2(w[i]), lo2);  // 0xFFFF where the column clips
              open |= ((~lt & 1u) | ((~lt >> 15) & 2u)) << (2 * i);
            }
          }
          nclip += 8u - __popc(open);
          *reinterpret_cast<uint4*>(buf + o) = make_uint4(jj2, jj2, jj2, jj2);
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u)  // constant indices once unrolled: w stays in registers
            if (o + u < nc) w[u >> 1] |= static_cast<uint32_t>(__ldg(xr + o + u)) << (16 * (u & 1));
          open = (1u << (nc - o)) - 1u;
        }
        while (open) {
          const int u = __ffs(open) - 1;
          open &= open - 1u;
          const uint32_t word = u < 2 ? w[0] : (u < 4 ? w[1] : (u < 6 ? w[2] : w[3]));
          settle(o + u, code16p((u & 1) ? (word >> 16) : (word & 0xFFFFu)));
        }
      }
    } else {
      for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
        uint32_t k8[8];
        samp_codes8<VEC>(a, row, cb + o, ce, k8);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (o + u < nc) settle(o + u, k8[u]);
      }
    }
    acc += static_cast<unsigned long long>(nclip) *
           static_cast<uint32_t>(__half2float(__ushort_as_half(ptab[0])) * 16777216.0f);
    acc = block_sum_u64_w0(acc, red);  // its barriers also complete this CTA's histogram and indices
    if (tid < C) st_cluster_u64(&xb[r], tid, acc);
    cluster_sync();
    if (tid < 32) {
      unsigned long long v = lane < C ? xb[lane] : 0ull;
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tid == 0) bcast = v;
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
      // The probability of an element is p(j) = fp16(table[S-1-j] / sum) of its table
      // index j alone, and p is non-increasing in j. The row's top-k by (p descending,
      // column ascending) lies in the union of every CTA's own top-k by the same order,
      // so each CTA selects its kl = min(k, columns) best columns locally (its k-th
      // smallest index j_k, the indices [j_lo, j_hi] whose probability equals p(j_k),
      // every column below j_lo and the first ties in column order), sorts them and
      // pushes them to the leader, which ranks the union.
      auto p16 = [&](int j) -> uint16_t {
        return __half_as_ushort(
            __float2half_rn(__fdiv_rn(__half2float(__ushort_as_half(ptab[a.size - 1 - j])), sum)));
      };
      const uint32_t k = static_cast<uint32_t>(a.k);
      const uint32_t kl = min(k, static_cast<uint32_t>(nc));
      if (kl > 0) {  // CTA-uniform
        int jk = jclip;
        if (fastb) {
          // C: the kl-th smallest offset from a block prefix over the counts (four
          // offsets per thread); clip index if fewer than kl columns are unclipped
          const int i0 = 4 * tid;
          uint32_t c4 = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) c4 += i0 + q < static_cast<int>(lw) ? icnt[i0 + q] : 0u;
          uint32_t incl = c4;
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
            scan[tid] = s2 - v;
            if (tid == 31) sel[0] = s2;  // unclipped columns of this CTA
          }
          __syncthreads();
          const uint32_t excl = scan[tid >> 5] + incl - c4;
          if (c4 > 0 && excl < kl && excl + c4 >= kl) {
            uint32_t run = excl;
            int istar = i0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              run += i0 + q < static_cast<int>(lw) ? icnt[i0 + q] : 0u;
              if (run >= kl) {
                istar = i0 + q;
                break;
              }
            }
            sel[2] = cj[istar];
          }
          __syncthreads();
          if (sel[0] >= kl) jk = static_cast<int>(sel[2]);
        } else {
          // C, D: j_k from the high-bit histogram, then the low 7 bits inside its bin
          if (tid < 32) {
            uint32_t below = 0;
            for (int i = lane; i < 256; i += 32) below += hist[i];
#pragma unroll
            for (int o = 16; o; o >>= 1) below += __shfl_xor_sync(0xffffffffu, below, o);
            uint32_t above = 0;
            const int b = below >= kl ? pick_bin_warp(hist, kl, &above) : -1;
            if (tid == 0) {
              sel[0] = static_cast<uint32_t>(b);
              sel[1] = above;
            }
          }
          __syncthreads();
          if (static_cast<int>(sel[0]) >= 0) {
            const int hb = 255 - static_cast<int>(sel[0]);
            const uint32_t above_hi = sel[1];
            for (int o = tid * 8; o < nc; o += 8 * kSampBlock) {
              uint32_t jv[8];
              buf_load8<VEC>(buf, o, nc, jv);
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int j = static_cast<int>(jv[u]);
                if (jv[u] != 0xFFFFu && j != jclip && (j >> 7) == hb) atomicAdd(&hist2[255 - (j & 127)], 1u);
              }
            }
            __syncthreads();
            if (tid < 32) {
              uint32_t above;
              const int lo = pick_bin_warp(hist2, kl - above_hi, &above);
              if (tid == 0) sel[2] = static_cast<uint32_t>((hb << 7) | (255 - lo));
            }
            __syncthreads();
            jk = static_cast<int>(sel[2]);
          }
        }
        __syncthreads();  // every thread has read j_k before sel[] is reused
        // [j_lo, j_hi]: 32-way searches of the monotone p, one warp each; the 32 indices
        // next to j_k first (a run of equal probabilities rarely reaches past them),
        // the whole range only if it does
        if (tid < 64) {
          const float pk = __half2float(__ushort_as_half(p16(jk)));
          if (tid < 32) {  // j_lo: first j in [0, j_k] with p(j) <= p(j_k)
            auto above = [&](uint32_t j) { return __half2float(__ushort_as_half(p16(static_cast<int>(j)))) > pk; };
            const uint32_t w0 = static_cast<uint32_t>(max(0, jk - 31));
            const uint32_t f = (w0 == 0 || above(w0)) ? warp_first_false(w0, static_cast<uint32_t>(jk), above)
                                                      : warp_first_false(0u, w0, above);
            if (tid == 0) sel[2] = f;
          } else {  // j_hi + 1: first j in [j_k, size] with p(j) < p(j_k) (size: past the table)
            auto tie = [&](uint32_t j) {
              return static_cast<int>(j) < a.size && __half2float(__ushort_as_half(p16(static_cast<int>(j)))) >= pk;
            };
            const uint32_t w1 = static_cast<uint32_t>(min(a.size, jk + 31));
            const uint32_t f = tie(w1) ? warp_first_false(w1, static_cast<uint32_t>(a.size), tie)
                                       : warp_first_false(static_cast<uint32_t>(jk), w1, tie);
            if (tid == 32) {
              sel[3] = f - 1u;
              sel[1] = p16(jk);
            }
          }
        }
        __syncthreads();
        const int jlo = static_cast<int>(sel[2]), jhi = static_cast<int>(sel[3]);
        // a column-buffer entry's table index (fast path: a code-table offset or 0xFFFF)
        auto jof = [&](uint32_t v) -> int {
          if (!fastb) return static_cast<int>(v);
          const int jt = cj[v < lw ? v : 0u];  // index always inside the table, sentinel or not
          return v == 0xFFFFu ? jclip : jt;
        };
        const uint32_t t = sel[1];  // fp16 bits of p(j_k)
        // E: contiguous column ranges of whole 8-column groups per thread, in column order
        const int sub = (((nc + kSampBlock - 1) / kSampBlock) + 7) & ~7;
        const int o0 = min(nc, tid * sub), o1 = min(nc, o0 + sub);
        uint32_t ties = 0;
        for (int o = o0; o < o1; o += 8) {
          uint32_t jv[8];
          buf_load8<VEC>(buf, o, o1, jv);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (o + u >= o1) break;
            const int j = jof(jv[u]);
            if (j < jlo) {  // p(j) > p(j_k): fewer than kl such columns here
              const uint32_t slot = atomicAdd(&lcn, 1u);
              if (slot < kSampMaxK)
                lc[slot] = (static_cast<unsigned long long>(p16(j)) << 32) | (0xFFFFFFFFull - (cb + o + u));
            } else if (j <= jhi) {  // p(j) == p(j_k)
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
        }
        __syncthreads();
        const uint32_t c_gt = min(lcn, kl);       // < kl by construction
        const uint32_t need = kl - c_gt;          // ties to take, the first ones by column
        uint32_t rank = scan[tid >> 5] + incl - ties;  // rank among this CTA's ties
        for (int o = o0; o < o1 && ties > 0 && rank < need; o += 8) {
          uint32_t jv[8];
          buf_load8<VEC>(buf, o, o1, jv);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (o + u < o1 && rank < need && jof(jv[u]) >= jlo && jof(jv[u]) <= jhi) {
              lc[c_gt + rank] = (static_cast<unsigned long long>(t) << 32) | (0xFFFFFFFFull - (cb + o + u));
              ++rank;
            }
          }
        }
        __syncthreads();
        // this CTA's kl keys, sorted (descending, distinct: the column is part of the
        // key), into the leader's list of this rank
        if (tid < static_cast<int>(kl)) {
          const unsigned long long key = lc[tid];
          uint32_t rk = 0;
          for (uint32_t i = 0; i < kl; ++i) rk += lc[i] > key ? 1u : 0u;
          st_cluster_u64(&xlist[r][rk], 0, key);
        }
      }
      if (tid == 0) st_cluster_u32(&xlen[r], 0, kl);
      cluster_sync();  // the leader holds every rank's sorted list
      if (leader) {
        // Merge the sorted lists pairwise, keeping the k largest keys of every merge: a
        // key's place in the merge is its place in its own list plus the number of
        // larger keys in the partner list (binary search; keys are distinct). Scratch:
        // the code table's space, free by now (at least 2 x 8 x 64 keys).
        unsigned long long* mbuf = reinterpret_cast<unsigned long long*>(ptab + a.lut_off);
        const unsigned long long* src = &xlist[0][0];
        const uint32_t* slen = xlen;
        __shared__ uint32_t mlen[2][kSampMaxCluster / 2];
        int lists = C, level = 0;
        while (lists > 1) {  // CTA-uniform
          unsigned long long* dst = mbuf + (level & 1) * (kSampMaxCluster / 2) * kSampMaxK;
          uint32_t* dlen = mlen[level & 1];
          const int L = tid / kSampMaxK, i = tid % kSampMaxK;
          if (L < lists && i < static_cast<int>(slen[L])) {
            const unsigned long long x = src[L * kSampMaxK + i];
            const int P = L ^ 1;
            uint32_t lo = 0;
            if (P < lists) {
              const unsigned long long* pl = src + P * kSampMaxK;
              uint32_t hi = slen[P];
              while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (pl[mid] > x)
                  lo = mid + 1;
                else
                  hi = mid;
              }
            }
            const uint32_t rk = static_cast<uint32_t>(i) + lo;
            if (rk < k) dst[(L >> 1) * kSampMaxK + rk] = x;
          }
          if (tid < (lists + 1) / 2) {
            const uint32_t l0 = slen[2 * tid], l1 = 2 * tid + 1 < lists ? slen[2 * tid + 1] : 0u;
            dlen[tid] = min(k, l0 + l1);
          }
          __syncthreads();
          src = dst;
          slen = dlen;
          lists = (lists + 1) / 2;
          ++level;
        }
        if (tid < static_cast<int>(k)) sorted[tid] = src[tid];
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
          // fp32 running sums in candidate order (eight loads in flight, then the adds)
          float total = 0.0f;
          for (uint32_t i0 = 0; i0 < k; i0 += 8) {
            float pv[8];
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q)
              pv[q] = i0 + q < k ? __half2float(__ushort_as_half(static_cast<uint16_t>(sorted[i0 + q] >> 32))) : 0.0f;
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q)
              if (i0 + q < k) total += pv[q];
          }
          uint32_t pick = k - 1;
          if (total > 0.0f) {
            const float target = u * total;
            float run = 0.0f;
            bool found = false;
            for (uint32_t i0 = 0; i0 < k && !found; i0 += 8) {
              float pv[8];
#pragma unroll
              for (uint32_t q = 0; q < 8; ++q)
                pv[q] = i0 + q < k ? __half2float(__ushort_as_half(static_cast<uint16_t>(sorted[i0 + q] >> 32))) : 0.0f;
#pragma unroll
              for (uint32_t q = 0; q < 8; ++q) {
                if (!found && i0 + q < k) {
                  run += pv[q];
                  if (run > target) {
                    pick = i0 + q;
                    found = true;
                  }
                }
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
// size (1 CTA of 1024 threads per SM; sizes above 8 are non-portable) fit at once.
constexpr int kSampMaxDevices = 64;
constexpr size_t kSampSmemMax = 184 * 1024;  // dynamic: the table, column buffer and code table
struct SampDevice {
  bool ready = false;
  int capacity[kSampMaxCluster + 1] = {};
};
static SampDevice g_samp_dev[kSampMaxDevices];
static std::once_flag g_samp_once[kSampMaxDevices];

template <bool VEC>
static bool samp_attrs() {
  if (cudaFuncSetAttribute(k_sample<VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kSampSmemMax)) != cudaSuccess ||
      cudaFuncSetAttribute(k_sample<VEC>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

static SampDevice& samp_device(int dev) {
  std::call_once(g_samp_once[dev], [dev] {
    SampDevice& sd = g_samp_dev[dev];
    if (!samp_attrs<true>() || !samp_attrs<false>()) return;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sd.capacity[1] = sms;
    for (int c = 2; c <= kSampMaxCluster; ++c) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, 1);
      cfg.blockDim = dim3(kSampBlock);
      cfg.dynamicSmemBytes = kSampSmemMax;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = c;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_sample<true>, &cfg) != cudaSuccess) {
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
  // a >= clip gives a / step > size - 1 in real numbers, so the fp32 quotient rounds to
  // at least size - 1 (representable) and the index clips: no division needed
  a.clip = static_cast<float>(static_cast<double>(size - 1) * static_cast<double>(a.step) * (1.0 + 0x1p-20));
  a.uniforms = uniforms;
  a.seed = seed;
  a.rng_state = rng_state;
  a.tokens = tokens;
  a.logprobs = logprobs;
  a.scratch = static_cast<uint16_t*>(workspace);
  a.err = dev_err;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kSampMaxDevices) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  SampDevice& sd = samp_device(dev);
  if (!sd.ready) return MB_ERR_LAUNCH;
  // cluster size: the largest C <= 16 whose N clusters are resident at once (one wave)
  int C = 1;
  for (int c = kSampMaxCluster; c >= 2; --c)
    if (sd.capacity[c] >= N) {
      C = c;
      break;
    }
  a.chunk = static_cast<int>((((static_cast<int64_t>(V) + C - 1) / C) + 7) / 8 * 8);
  const size_t tab_bytes = static_cast<size_t>((size + 7) & ~7) * sizeof(uint16_t);
  // the code table's space doubles as the leader's merge scratch: keep at least 8 KB
  a.buf_smem = tab_bytes + static_cast<size_t>(a.chunk) * sizeof(uint16_t) + 8192 <= kSampSmemMax ? 1 : 0;
  // the rest of the budget holds the code -> index table (up to every fp16 code)
  a.lut_off = static_cast<int>(tab_bytes / sizeof(uint16_t)) + (a.buf_smem ? a.chunk : 0);
  a.lut_cap = std::min(65536, static_cast<int>(kSampSmemMax / sizeof(uint16_t)) - a.lut_off) & ~7;
  if (a.lut_cap < 0) a.lut_cap = 0;
  const size_t smem = (static_cast<size_t>(a.lut_off) + a.lut_cap) * sizeof(uint16_t);
  // 16-byte loads of whole 8-column groups: every row and chunk starts 16-byte aligned
  const bool vec = V % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(workspace) & 15) == 0;
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
  if ((vec ? cudaLaunchKernelEx(&cfg, k_sample<true>, a) : cudaLaunchKernelEx(&cfg, k_sample<false>, a)) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return launch_status();
}

}  // extern "C"
