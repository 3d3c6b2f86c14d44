// Fused INT4 super-block batched GEMM for B200 (sm_100a):
//   out[N, M] (fp16) = act[N, K] (fp16) x dequant(sb)[K, M], fp32 accumulation.
//
// Replaces the reference's batched_gemm entry point (Metal batched_gemm_simdgroup /
// fused_batched_gemm_int4, antigravity-engine/src/shaders/batched_gemm.metal:74-169;
// CPU form `activations @ W`, batch_generator.py:290). The weight stream is the
// reference's 144-byte super-block format, read in place.
//
// Design (weight-streaming, HBM bound):
//  * Work = (strip of 256 columns = one super-block per row) x (16-row k slices),
//    split evenly over a persistent grid in strip-major order (stream-K), so every
//    SM streams the same number of weight bytes whatever K, M and the SM count are.
//  * One producer thread per CTA issues 2-D TMA tile loads (cp.async.bulk.tensor):
//    16 rows x 144 B of super-blocks per slice (L2 evict-first) and a 64-wide k tile
//    of the activations (128-byte swizzle, L2 evict-last) into a multi-stage
//    shared-memory ring guarded by mbarriers.
//  * Programmatic dependent launch: weights never depend on the previous kernel, so
//    the producer prefetches its first stages BEFORE griddepcontrol.wait; only the
//    activation loads and all global writes wait for the previous grid.
//  * Four consumer warps expand nibbles straight into mma.m16n8k16 A fragments in
//    registers (byte permute + magic-exponent fp16 conversion + one fp16 multiply by
//    the group scale, bit-exact with the reference dequant) and accumulate in fp32.
//    The batch (padded to 8/16/32 rows) is the MMA n dimension.
//  * Split-K partial sums go to an fp32 workspace in L2 with vector reductions; the
//    last CTA to finish a strip (arrival counter) converts it to fp16 and re-zeroes
//    the workspace, so the workspace is clean for the next call.
#include <algorithm>

#include "common.cuh"

namespace mb {

constexpr int kSB = 144;                 // bytes per super-block
constexpr int kStripCols = 256;          // columns per strip (one super-block per row)
constexpr int kSliceRows = 16;           // k rows per MMA slice
constexpr int kSliceBytes = kSliceRows * kSB;  // 2304, a multiple of 128
constexpr int kSlicesPerStage = 4;
constexpr int kStageWBytes = kSlicesPerStage * kSliceBytes;  // 9216
constexpr int kConsumerWarps = 4;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kRedStride = 256 + 4;        // padded fp32 row of the reduction tile

struct GemmArgs {
  uint16_t* out;        // [N, M] fp16
  float* ws;            // [N, M] fp32 partial sums, zero between calls
  uint32_t* counters;   // [nstrips]
  uint32_t* err;        // device error word
  int N, K, M;
  int KS;               // k slices per strip
  long long U;          // total units = nstrips * KS
  int G;                // grid size
};

template <int NT>
struct Cfg {
  static constexpr int kStages = (NT == 4) ? 4 : 6;
  static constexpr int kXBytes = 8 * NT * 128;  // [8*NT rows][64 fp16], 128B-swizzled
  static constexpr int kRedBytes = 8 * NT * kRedStride * 4;
  static constexpr int kSmem = 1024 + kStages * kXBytes + kStages * kStageWBytes + kRedBytes + 2 * kStages * 8 + 16;
};

struct StageIter {
  long long u, end;
  int KS;
  __device__ __forceinline__ bool next(int& strip, int& sl, int& n) {
    if (u >= end) return false;
    strip = static_cast<int>(u / KS);
    sl = static_cast<int>(u - static_cast<long long>(strip) * KS);
    long long m = KS - sl;
    if (end - u < m) m = end - u;
    if (m > kSlicesPerStage) m = kSlicesPerStage;
    n = static_cast<int>(m);
    u += n;
    return true;
  }
};

__device__ __forceinline__ long long range_begin(long long c, long long U, int G) { return (c * U) / G; }

__device__ __forceinline__ int cta_of(long long u, long long U, int G) {
  long long c = (u * G) / U;
  while (c + 1 < G && range_begin(c + 1, U, G) <= u) ++c;
  while (c > 0 && range_begin(c, U, G) > u) --c;
  return static_cast<int>(c);
}

__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

template <int NW>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[NW]) {
  if constexpr (NW == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (NW == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

// One 16-row k slice for this thread's column run.
//   wsl: slice base (16 rows x 144 B); xt: stage activation tile; j: slice index in stage
//   colbyte: byte offset of the thread's first nibble in a row; grp: its scale group.
// Thread (g4 = lane/4, t4 = lane%4) owns rows 2t4, 2t4+1, 2t4+8, 2t4+9 of the slice
// (the k positions of the m16n8k16 A fragment) and MR consecutive columns; m16 tile
// i of the warp maps fragment row g4 to column 2i and row g4+8 to column 2i+1 of the
// thread's run, so each nibble byte feeds one tile.
template <int NT>
__device__ __forceinline__ void consume_slice(const uint8_t* wsl, const uint8_t* xt, int j, int g4, int t4, int colbyte,
                                              int grp, float (&acc)[16 / NT][NT][4]) {
  constexpr int NW = 4 / NT;  // 32-bit nibble words per row per thread
  const uint8_t* r0 = wsl + (2 * t4) * kSB;
  const uint8_t* r1 = r0 + kSB;
  const uint8_t* r2 = r0 + 8 * kSB;
  const uint8_t* r3 = r2 + kSB;
  uint32_t w0[NW], w1[NW], w2[NW], w3[NW];
  lds_words<NW>(r0 + colbyte, w0);
  lds_words<NW>(r1 + colbyte, w1);
  lds_words<NW>(r2 + colbyte, w2);
  lds_words<NW>(r3 + colbyte, w3);
  const uint32_t s01 = lds_u16(r0 + 2 * grp) | (lds_u16(r1 + 2 * grp) << 16);
  const uint32_t s23 = lds_u16(r2 + 2 * grp) | (lds_u16(r3 + 2 * grp) << 16);
  uint32_t bf[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint8_t* xr = xt + (nt * 8 + g4) * 128 + 4 * t4;
    bf[nt][0] = lds_u32(xr + (((2 * j) ^ g4) << 4));
    bf[nt][1] = lds_u32(xr + (((2 * j + 1) ^ g4) << 4));
  }
#pragma unroll
  for (int v = 0; v < NW; ++v) {
    const uint32_t p01l = prmt(w0[v], w1[v], 0x5410u), p01h = prmt(w0[v], w1[v], 0x7632u);
    const uint32_t p23l = prmt(w2[v], w3[v], 0x5410u), p23h = prmt(w2[v], w3[v], 0x7632u);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t q01 = ((b & 2) ? p01h : p01l) >> (8 * (b & 1));
      const uint32_t q23 = ((b & 2) ? p23h : p23l) >> (8 * (b & 1));
      uint32_t a0, a1, a2, a3;
      nibbles_to_half2(q01, a0, a1);
      nibbles_to_half2(q23, a2, a3);
      a0 = hmul2(a0, s01);
      a1 = hmul2(a1, s01);
      a2 = hmul2(a2, s23);
      a3 = hmul2(a3, s23);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816(acc[4 * v + b][nt], a0, a1, a2, a3, bf[nt][0], bf[nt][1]);
    }
  }
}

template <int NT>
__device__ __forceinline__ void store_half4(uint16_t* dst, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}

// Strip epilogue: reduce the four warps' partial sums in shared memory, then either
// write fp16 directly (this CTA covered the whole strip) or add into the fp32
// workspace; the last arriving CTA converts the strip to fp16 and re-zeroes it.
template <int NT>
__device__ __forceinline__ void strip_epilogue(const GemmArgs& p, int strip, float (&acc)[16 / NT][NT][4],
                                               float* red, int* flag, int ctid, int g4, int t4, int mbt) {
  constexpr int MT = 16 / NT;
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int n = nt * 8 + 2 * t4 + (c & 1);
        const int col = mbt + 2 * i + (c >> 1);
        if (n < p.N) atomicAdd(&red[n * kRedStride + col], acc[i][nt][c]);
        acc[i][nt][c] = 0.0f;
      }
  named_bar_sync(1, kConsumers);

  const long long s0 = static_cast<long long>(strip) * p.KS;
  const int first = cta_of(s0, p.U, p.G);
  const int last = cta_of(s0 + p.KS - 1, p.U, p.G);
  const int nvec = p.N * (kStripCols / 4);
  const size_t colbase = static_cast<size_t>(strip) * kStripCols;

  if (first == last) {  // sole owner of the strip
    for (int idx = ctid; idx < nvec; idx += kConsumers) {
      const int n = idx >> 6, c4 = (idx & 63) * 4;
      float4* rp = reinterpret_cast<float4*>(red + n * kRedStride + c4);
      const float4 v = *rp;
      *rp = make_float4(0.f, 0.f, 0.f, 0.f);
      store_half4<NT>(p.out + static_cast<size_t>(n) * p.M + colbase + c4, v);
    }
    named_bar_sync(1, kConsumers);
    return;
  }

  for (int idx = ctid; idx < nvec; idx += kConsumers) {
    const int n = idx >> 6, c4 = (idx & 63) * 4;
    float4* rp = reinterpret_cast<float4*>(red + n * kRedStride + c4);
    const float4 v = *rp;
    *rp = make_float4(0.f, 0.f, 0.f, 0.f);
    red_add_v4(p.ws + static_cast<size_t>(n) * p.M + colbase + c4, v.x, v.y, v.z, v.w);
  }
  __threadfence();
  named_bar_sync(1, kConsumers);
  if (ctid == 0) {
    const uint32_t old = atomicAdd(&p.counters[strip], 1u);
    *flag = (old == static_cast<uint32_t>(last - first)) ? 1 : 0;
  }
  named_bar_sync(1, kConsumers);
  if (*flag) {
    __threadfence();
    for (int idx = ctid; idx < nvec; idx += kConsumers) {
      const int n = idx >> 6, c4 = (idx & 63) * 4;
      float4* gp = reinterpret_cast<float4*>(p.ws + static_cast<size_t>(n) * p.M + colbase + c4);
      const float4 v = __ldcg(gp);
      __stcg(gp, make_float4(0.f, 0.f, 0.f, 0.f));
      store_half4<NT>(p.out + static_cast<size_t>(n) * p.M + colbase + c4, v);
    }
    if (ctid == 0) atomicExch(&p.counters[strip], 0u);
  }
  named_bar_sync(1, kConsumers);
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tma(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, const GemmArgs p) {
  using C = Cfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint8_t* wsm = xs + S * C::kXBytes;
  float* red = reinterpret_cast<float*>(wsm + S * kStageWBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + C::kRedBytes);
  uint64_t* empty = full + S;
  int* flag = reinterpret_cast<int*>(empty + S);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long b0 = range_begin(blockIdx.x, p.U, p.G);
  const long long b1 = range_begin(blockIdx.x + 1, p.U, p.G);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kConsumerWarps);
    }
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 8 * NT * kRedStride; i += kThreads) red[i] = 0.0f;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane != 0) return;
    const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
    StageIter it{b0, b1, p.KS};
    int strip, sl, n;
    int pre_sl[S];
    int npre = 0;
    while (npre < S && it.next(strip, sl, n)) {
      mbar_expect_tx(full + npre, n * kSliceBytes + C::kXBytes);
      for (int j = 0; j < n; ++j)
        tma_load_2d(wsm + npre * kStageWBytes + j * kSliceBytes, &wmap, full + npre, strip * kSB,
                    (sl + j) * kSliceRows, pol_w);
      pre_sl[npre++] = sl;
    }
    pdl_wait();  // activations may be written by the previous grid
    for (int s = 0; s < npre; ++s) tma_load_2d(xs + s * C::kXBytes, &xmap, full + s, pre_sl[s] * kSliceRows, 0, pol_x);
    int i = npre;
    while (it.next(strip, sl, n)) {
      const int s = i % S;
      if (!mbar_wait(empty + s, ((i / S) - 1) & 1)) atomicOr(p.err, MB_DEVERR_TIMEOUT);
      mbar_expect_tx(full + s, n * kSliceBytes + C::kXBytes);
      for (int j = 0; j < n; ++j)
        tma_load_2d(wsm + s * kStageWBytes + j * kSliceBytes, &wmap, full + s, strip * kSB, (sl + j) * kSliceRows,
                    pol_w);
      tma_load_2d(xs + s * C::kXBytes, &xmap, full + s, sl * kSliceRows, 0, pol_x);
      ++i;
    }
    return;
  }

  // ---------------- consumers ----------------
  constexpr int MR = 32 / NT;  // columns per thread per row
  constexpr int MT = MR / 2;   // m16 tiles per warp
  const int g4 = lane >> 2, t4 = lane & 3;
  const int mpart = warp % NT;
  const int slice0 = warp / NT;
  constexpr int slice_step = kConsumerWarps / NT;
  const int mbt = mpart * (kStripCols / NT) + g4 * MR;
  const int colbyte = 16 + mbt / 2;
  const int grp = mbt / 32;
  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][nt][c] = 0.0f;

  pdl_wait();  // all global writes below happen after the previous grid completed
  StageIter it{b0, b1, p.KS};
  int strip, sl, n, i = 0;
  while (it.next(strip, sl, n)) {
    const int s = i % S;
    if (!mbar_wait(full + s, (i / S) & 1) && lane == 0) atomicOr(p.err, MB_DEVERR_TIMEOUT);
    const uint8_t* wst = wsm + s * kStageWBytes;
    const uint8_t* xt = xs + s * C::kXBytes;
    for (int j = slice0; j < n; j += slice_step) consume_slice<NT>(wst + j * kSliceBytes, xt, j, g4, t4, colbyte, grp, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    ++i;
    if (it.u == it.end || (it.u % p.KS) == 0) strip_epilogue<NT>(p, strip, acc, red, flag, threadIdx.x, g4, t4, mbt);
  }
}

// ---------------------------------------------------------------------------
// Generic path (any M with K*M % 256 == 0; K not a multiple of 8): one thread per
// output column, flat super-block indexing as in fused_batched_gemm_int4
// (batched_gemm.metal:146-155), activations staged in shared memory. Correct for
// every shape; the TMA path above is the fast one.
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(128) k_gemm_generic(const uint16_t* __restrict__ act, const uint8_t* __restrict__ sb,
                                                      uint16_t* __restrict__ out, int N, int K, int M) {
  constexpr int KC = 64;
  __shared__ float xs[NB][KC];
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  float acc[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n] = 0.0f;
  pdl_wait();
  for (int k0 = 0; k0 < K; k0 += KC) {
    __syncthreads();
    for (int t = threadIdx.x; t < NB * KC; t += blockDim.x) {
      const int n = t / KC, kk = t % KC;
      xs[n][kk] = (n < N && k0 + kk < K) ? __half2float(__ushort_as_half(act[static_cast<size_t>(n) * K + k0 + kk])) : 0.0f;
    }
    __syncthreads();
    if (m < M) {
      const int kend = min(KC, K - k0);
      for (int kk = 0; kk < kend; ++kk) {
        const long long flat = static_cast<long long>(k0 + kk) * M + m;
        const uint8_t* b = sb + (flat >> 8) * kSB;
        const int e = static_cast<int>(flat & 255);
        const int byte = __ldg(b + 16 + (e >> 1));
        const int q = ((e & 1) ? (byte >> 4) : (byte & 15)) - 8;
        const __half s = __ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(b) + (e >> 5)));
        const float w = __half2float(__hmul(__int2half_rn(q), s));
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(xs[n][kk], w, acc[n]);
      }
    }
  }
  if (m < M)
#pragma unroll
    for (int n = 0; n < NB; ++n)
      if (n < N) out[static_cast<size_t>(n) * M + m] = __half_as_ushort(__float2half_rn(acc[n]));
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static constexpr size_t kWsHeader = 256;

static inline size_t ws_counters_bytes(int M) {
  const size_t nstrips = (static_cast<size_t>(M) + kStripCols - 1) / kStripCols;
  return (nstrips * 4 + 255) / 256 * 256;
}

static inline bool tma_path_ok(const void* act, const void* sb, int K, int M) {
  return M % kStripCols == 0 && K % 8 == 0 && aligned(act, 16) && aligned(sb, 16);
}

// Resident CTAs per SM for k_gemm_tma<NT> on the current device (capped at 2 so a
// dependent grid launched with PDL finds room to start its prefetch). The first call
// on a device also raises the kernel's dynamic shared-memory limit there.
template <int NT>
static int blocks_per_sm() {
  static int per_dev[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (per_dev[dev] == 0) {
    if (cudaFuncSetAttribute(k_gemm_tma<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<NT>::kSmem) !=
        cudaSuccess)
      return 0;
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_gemm_tma<NT>, kThreads, Cfg<NT>::kSmem) != cudaSuccess)
      return 0;
    per_dev[dev] = std::max(1, std::min(b, 2));
  }
  return per_dev[dev];
}

template <int NT>
static int grid_size(long long U) {
  const int b = blocks_per_sm<NT>();
  if (b == 0) return 0;
  const long long g = static_cast<long long>(b) * sm_count();
  return static_cast<int>(std::min<long long>(g, U));
}

template <int NT>
static int launch_tma(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, uint8_t* ws,
                      cudaStream_t st) {
  CUtensorMap wmap, xmap;
  const uint64_t row_bytes = static_cast<uint64_t>(M / kStripCols) * kSB;
  if (!encode_tmap_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, sb, row_bytes, K, row_bytes, kSB, kSliceRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
    return MB_ERR_LAUNCH;
  if (!encode_tmap_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, K, N, static_cast<uint64_t>(K) * 2, 64, 8 * NT,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return MB_ERR_LAUNCH;
  GemmArgs a;
  a.out = out;
  a.err = reinterpret_cast<uint32_t*>(ws);
  a.counters = reinterpret_cast<uint32_t*>(ws + kWsHeader);
  a.ws = reinterpret_cast<float*>(ws + kWsHeader + ws_counters_bytes(M));
  a.N = N;
  a.K = K;
  a.M = M;
  a.KS = (K + kSliceRows - 1) / kSliceRows;
  a.U = static_cast<long long>(M / kStripCols) * a.KS;
  a.G = grid_size<NT>(a.U);
  if (a.G <= 0) return MB_ERR_LAUNCH;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg<NT>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_gemm_tma<NT>, wmap, xmap, a) != cudaSuccess) return MB_ERR_LAUNCH;
  return launch_status();
}

static int launch_generic(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, cudaStream_t st) {
  const dim3 grid((M + 127) / 128);
  if (N <= 8)
    k_gemm_generic<8><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  else if (N <= 16)
    k_gemm_generic<16><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  else
    k_gemm_generic<32><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  return launch_status();
}

}  // namespace mb

using namespace mb;

extern "C" {

size_t mb_int4_gemm_workspace_size(int32_t N, int32_t K, int32_t M) {
  (void)K;
  if (N < 1 || M < 1) return 0;
  const size_t rows = static_cast<size_t>(std::min(N, 32));
  return kWsHeader + ws_counters_bytes(M) + rows * static_cast<size_t>(M) * 4;
}

int32_t mb_int4_gemm(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (!act || !sb || !out) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tma = tma_path_ok(act, sb, K, M);
  if (tma) {
    if (!workspace) return MB_ERR_NULL;
    if (!aligned(workspace, 256) || !aligned(out, 8)) return MB_ERR_ALIGN;
    if (workspace_bytes < mb_int4_gemm_workspace_size(N, K, M)) return MB_ERR_WORKSPACE;
  }
  for (int r0 = 0; r0 < N; r0 += 32) {
    const int nb = std::min(32, N - r0);
    const uint16_t* a = act + static_cast<size_t>(r0) * K;
    uint16_t* o = out + static_cast<size_t>(r0) * M;
    int rc;
    if (tma && aligned(a, 16)) {
      uint8_t* ws = static_cast<uint8_t*>(workspace);
      if (nb <= 8)
        rc = launch_tma<1>(a, sb, o, nb, K, M, ws, st);
      else if (nb <= 16)
        rc = launch_tma<2>(a, sb, o, nb, K, M, ws, st);
      else
        rc = launch_tma<4>(a, sb, o, nb, K, M, ws, st);
    } else {
      rc = launch_generic(a, sb, o, nb, K, M, st);
    }
    if (rc != MB_OK) return rc;
  }
  return MB_OK;
}

int32_t mb_int4_gemm_device_status(void* workspace, uint32_t* status_out, void* stream) {
  if (!workspace || !status_out) return MB_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status_out, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return MB_ERR_LAUNCH;
  if (cudaMemsetAsync(workspace, 0, 4, st) != cudaSuccess) return MB_ERR_LAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return MB_ERR_LAUNCH;
  return MB_OK;
}

}  // extern "C"
