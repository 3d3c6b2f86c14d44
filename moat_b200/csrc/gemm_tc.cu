// INT4 super-block GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   out[N, M] (fp16) = act[N, K] (fp16) x dequant(sb)[K, M], fp32 accumulation,
//
// for M % 256 == 0 and K % 8 == 0 (the reference's batched_gemm entry point,
// antigravity-engine/src/shaders/batched_gemm.metal:74-169, on its 144-byte
// super-block stream read in place).
//
// Per CTA: one strip of 256 output columns (one super-block per weight row) and a
// 1/Ck slice of K; the Ck CTAs of a strip form a thread-block cluster and reduce
// their partial sums through distributed shared memory.
//
//  * warp 0: one thread streams the strip's rows with 3-D TMA tile loads (144-byte
//    rows, 128 rows per stage) into a ring of shared-memory stages. Weights do not
//    depend on the previous kernel, so the ring is filled before the programmatic
//    dependent launch wait.
//  * warps 2.. (G groups of four, one warp per TMEM lane quarter): expand nibbles to
//    fp16 with the exact magic-exponent conversion and one rounding multiply by the
//    group scale (bit-identical to the reference dequant) and store each 16-row
//    K step as two 128 x 16 A tiles in tensor memory (tcgen05.st.16x256b).
//    The dequant never touches the activations, so it also runs ahead of the wait.
//  * warp 1: allocates TMEM; after griddepcontrol.wait, one thread loads this CTA's
//    activation slice with TMA in the canonical K-major layout and issues the MMAs
//    (M = 128 columns, N = batch padded to 16 / 32, K = 16) that accumulate both
//    128-column halves of the strip in TMEM; tcgen05.commit frees each A tile.
//  * epilogue: one dequant group reads the accumulators (tcgen05.ld), the cluster
//    sums the Ck partial tiles in a fixed order (deterministic) and stores fp16.
//
// All waits are bounded (MB_DEVERR_TIMEOUT in the optional error word).
#include <algorithm>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace mb {
namespace tc {

constexpr int kSB = 144;                          // bytes per super-block (= per weight row of a strip)
constexpr int kStepRows = 16;                     // k rows per MMA
constexpr int kStageSteps = 8;                    // MMA K steps per TMA stage
constexpr int kStageRows = kStageSteps * kStepRows;
constexpr int kStageBytes = kStageRows * kSB;     // 18432
constexpr int kMaxStages = 8;

struct Params {
  uint16_t* out;
  uint32_t* err;
  int N, K, M;
  int KS;       // K steps, ceil(K / 16)
  int Ck;       // CTAs per cluster (K split)
  int S;        // stage ring depth
  int xoff;     // shared-memory offset of the activation tile
  int xblocks;  // 64-wide k blocks of the activation tile
  int tcols;    // TMEM columns allocated
  int baroff;   // shared-memory offset of the barriers
};

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

__device__ __forceinline__ void st_half2(uint16_t* dst, float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  *reinterpret_cast<__half2*>(dst) = h;
}

template <int NP, int G, int NB>
__global__ void __launch_bounds__((2 + 4 * G) * 32, 2)
    k_gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = static_cast<int>(blockIdx.x) % p.Ck;  // rank in the cluster = K part
  const int strip = static_cast<int>(blockIdx.x) / p.Ck;
  const int ks0 = static_cast<int>((static_cast<long long>(q) * p.KS) / p.Ck);
  const int ks1 = static_cast<int>((static_cast<long long>(q + 1) * p.KS) / p.Ck);
  const int nks = ks1 - ks0;
  const int nst = (nks + kStageSteps - 1) / kStageSteps;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kMaxStages;
  uint64_t* freeb = empty + kMaxStages;  // [G][NB]: MMAs reading an A buffer are done
  uint64_t* dfull = freeb + G * NB;       // [G]: a group's last MMA is done
  uint64_t* xfull = dfull + G;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(xfull + 1);
  uint8_t* xs = smem + p.xoff;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 4 * kStageSteps);
    }
    for (int i = 0; i < G * NB; ++i) mbar_init(freeb + i, 1);
    for (int g = 0; g < G; ++g) mbar_init(dfull + g, 1);
    mbar_init(xfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, static_cast<uint32_t>(p.tcols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // TMEM columns: A buffers [0, 16 G NB); group g accumulates strip half a in
  // [dcol + (2 g + a) NP, dcol + (2 g + a + 1) NP)
  const uint32_t dcol = G * NB * 16;
  pdl_launch_dependents();

  // Every wait is bounded; after its first timeout a thread waits no more, so the
  // kernel always ends within a few wait budgets.
  bool timeout = false;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (!timeout && !mbar_wait(bar, parity)) timeout = true;
  };
  if (warp == 0) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int st = 0; st < nst; ++st) {
        const int s = st % p.S;
        if (st >= p.S) wait(empty + s, ((st / p.S) - 1) & 1);
        mbar_expect_tx(full + s, kStageBytes);
        tma_load_3d(smem + s * kStageBytes, &wmap, full + s, 0, strip, (ks0 + st * kStageSteps) * kStepRows, pol);
      }
      // no copy may still be landing when the CTA leaves
      for (int st = nst > p.S ? nst - p.S : 0; st < nst; ++st) wait(full + st % p.S, (st / p.S) & 1);
    }
  } else if (warp == 1) {
    // ---------------- activations: 64-wide k blocks, 128-byte swizzle ----------------
    if (lane == 0) {
      pdl_wait();  // activations may be written by the previous kernel
      mbar_expect_tx(xfull, static_cast<uint32_t>(p.xblocks * NP * 128));
      const uint64_t polx = policy_evict_last();
      for (int b = 0; b < p.xblocks; ++b) tma_load_2d(xs + b * NP * 128, &xmap, xfull, 16 * ks0 + 64 * b, 0, polx);
      wait(xfull, 0);  // nothing may still be landing when the CTA leaves
    }
  } else {
    // ---------------- dequant into TMEM A tiles, one MMA stream per group ----------------
    const int grp = (warp - 2) >> 2;
    const int qq = warp & 3;  // TMEM lane quarter this warp may access
    const int g4 = lane >> 2, t4 = lane & 3;
    const bool issuer = ((warp - 2) & 3) == 0 && lane == 0;
    const int nboff = 16 + 32 * qq + 4 * g4;     // this thread's 4 nibble bytes (8 columns) in a row
    const int scoff = 2 * (2 * qq + (g4 >> 2));  // their group scale
    const uint32_t lanebase = tbase + (static_cast<uint32_t>(32 * qq) << 16);
    const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NP >> 3) << 17) | (8u << 24);
    const uint32_t xaddr = smem_u32(xs);
    const uint32_t dg = tbase + dcol + static_cast<uint32_t>(2 * grp * NP);
    bool first = true;
    for (int kl = grp; kl < nks; kl += G) {
      const int i = (kl - grp) / G, b = i % NB, u = i / NB;
      const int st = kl / kStageSteps, s = st % p.S;
      wait(full + s, (st / p.S) & 1);
      // rows 4 t4 .. 4 t4 + 3 of the K step: thread writes k positions 4 t4 .. 4 t4 + 3
      const uint8_t* rp = smem + s * kStageBytes + ((kl % kStageSteps) * kStepRows + 4 * t4) * kSB;
      const uint32_t w0 = lds32(rp + nboff), w1 = lds32(rp + kSB + nboff);
      const uint32_t w2 = lds32(rp + 2 * kSB + nboff), w3 = lds32(rp + 3 * kSB + nboff);
      const uint32_t s01 = lds16(rp + scoff) | (lds16(rp + kSB + scoff) << 16);
      const uint32_t s23 = lds16(rp + 2 * kSB + scoff) | (lds16(rp + 3 * kSB + scoff) << 16);
      // byte j of (row a, row a+1) side by side: the magic conversion of bytes 0 / 2
      // then yields k pairs (row a, row a+1) for the low and the high nibble column
      const uint32_t p01l = prmt(w0, w1, 0x5410u), p01h = prmt(w0, w1, 0x7632u);
      const uint32_t p23l = prmt(w2, w3, 0x5410u), p23h = prmt(w2, w3, 0x7632u);
      uint32_t r[4][4];  // [byte j][lo nibble rows 0-1, lo rows 2-3, hi rows 0-1, hi rows 2-3]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t q01 = ((j & 2) ? p01h : p01l) >> (8 * (j & 1));
        const uint32_t q23 = ((j & 2) ? p23h : p23l) >> (8 * (j & 1));
        uint32_t lo01, hi01, lo23, hi23;
        nibbles_to_half2(q01, lo01, hi01);
        nibbles_to_half2(q23, lo23, hi23);
        r[j][0] = hmul2(lo01, s01);
        r[j][1] = hmul2(lo23, s23);
        r[j][2] = hmul2(hi01, s01);
        r[j][3] = hmul2(hi23, s23);
      }
      // the buffer's previous MMAs must be done before it is overwritten
      if (u >= 1) {
        wait(freeb + grp * NB + b, (u - 1) & 1);
        tc_fence_after();
      }
      __syncwarp();
      // lanes 0-15 of the quarter take bytes 0 / 2 (A tile 0 / 1), lanes 16-31 bytes 1 / 3:
      // TMEM lane 32 qq + 16 (j & 1) + 8 hi + g4 of A tile j >> 1 is output column
      // 64 qq + 8 g4 + 2 j + hi of the strip
      const uint32_t acol = static_cast<uint32_t>((grp * NB + b) * 16);
      tmem_st_16x256b_x2(lanebase + acol, r[0][0], r[0][1], r[0][2], r[0][3], r[2][0], r[2][1], r[2][2], r[2][3]);
      tmem_st_16x256b_x2(lanebase + (16u << 16) + acol, r[1][0], r[1][1], r[1][2], r[1][3], r[3][0], r[3][1], r[3][2],
                         r[3][3]);
      tmem_wait_st();
      tc_fence_before();
      named_bar_sync(1 + grp, 128);  // the group's four quarters of the A tiles are written
      if (lane == 0) mbar_arrive(empty + s);
      if (issuer) {
        if (first) wait(xfull, 0);
        first = false;
        tc_fence_after();
        // K step kl of the activations: 64-wide block kl / 4, 32-byte offset (kl % 4) inside
        // the 128-byte swizzled rows; 8-row groups 1024 bytes apart
        const uint32_t xa = xaddr + static_cast<uint32_t>((kl >> 2) * NP * 128 + (kl & 3) * 32);
        const uint64_t bdesc = smem_desc_sw128_kmajor(xa);
        tc_mma_f16_ts(dg, tbase + acol, bdesc, idesc, i > 0 ? 1u : 0u);
        tc_mma_f16_ts(dg + NP, tbase + acol + 8, bdesc, idesc, i > 0 ? 1u : 0u);
        tc_commit(freeb + grp * NB + b);
        if (kl + G >= nks) tc_commit(dfull + grp);
      }
    }
    if (grp == 0) {
      // ---------------- epilogue: sum the groups' accumulators -> shared [NP][256] fp32 ----------------
      for (int g = 0; g < G; ++g)
        if (g < nks) wait(dfull + g, 0);
      __syncwarp();
      tc_fence_after();
      pdl_wait();
      float* part = reinterpret_cast<float*>(smem);  // the stage ring is drained by now
      const int beta = (lane >> 4) & 1, hi = (lane >> 3) & 1, gg = lane & 7;
      const int ng = nks < G ? nks : G;
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const int col = 64 * qq + 8 * gg + 4 * a + 2 * beta + hi;
#pragma unroll
        for (int h = 0; h < NP / 16; ++h) {
          float acc[16];
#pragma unroll
          for (int n = 0; n < 16; ++n) acc[n] = 0.0f;
          for (int g = 0; g < ng; ++g) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(lanebase + dcol + (2 * g + a) * NP + 16 * h, v);
            tmem_wait_ld();
#pragma unroll
            for (int n = 0; n < 16; ++n) acc[n] += __uint_as_float(v[n]);
          }
#pragma unroll
          for (int n = 0; n < 16; ++n) part[(16 * h + n) * 256 + col] = acc[n];
        }
      }
      tc_fence_before();
    }
  }
  __syncthreads();

  // ---- final sums: this CTA writes columns [q * 256 / Ck, (q + 1) * 256 / Ck) ----
  if (p.Ck > 1) cluster_sync();
  {
    const int cw = 256 / p.Ck, half = cw / 2;
    const int cb = q * cw;
    const float* part = reinterpret_cast<const float*>(smem);
    const uint32_t pbase = smem_u32(smem);
    uint16_t* ob = p.out + static_cast<size_t>(strip) * 256;
    for (int e = threadIdx.x; e < p.N * half; e += blockDim.x) {
      const int n = e / half, col = cb + 2 * (e - n * half);
      float lo = 0.0f, hi = 0.0f;
      if (p.Ck == 1) {
        lo = part[n * 256 + col];
        hi = part[n * 256 + col + 1];
      } else {
        const uint32_t off = pbase + 4u * static_cast<uint32_t>(n * 256 + col);
        for (int c = 0; c < p.Ck; ++c) {
          const uint32_t a = mapa_shared(off, static_cast<uint32_t>(c));
          lo += ld_shared_cluster_f32(a);
          hi += ld_shared_cluster_f32(a + 4);
        }
      }
      st_half2(ob + static_cast<size_t>(n) * p.M + col, lo, hi);
    }
  }
  if (p.Ck > 1) cluster_sync();  // peers may still read this CTA's partial tile

  if (warp == 1) {
    // no MMA may still use TMEM (the epilogue waited for every group's last one)
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, static_cast<uint32_t>(p.tcols));
  }
  if (timeout && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// (groups, A buffers per group): 4 x 2 at N <= 16, 3 x 1 at N <= 32, so that the A
// buffers plus one accumulator pair per group fit 256 TMEM columns (two CTAs per SM)
template <int NP> struct Cfg;
template <> struct Cfg<16> { static constexpr int G = 4, NB = 2; };
template <> struct Cfg<32> { static constexpr int G = 3, NB = 1; };

constexpr int kSmemBudget = 110 * 1024;  // two CTAs per SM: this call's and the next call's

bool plan(int N, int K, int M, int sms, TcPlan* pl) {
  *pl = TcPlan();
  if (N < 1 || N > 32 || M % 256 != 0 || K % 8 != 0) return false;
  const int NP = N <= 16 ? 16 : 32;
  const int G = NP == 16 ? Cfg<16>::G : Cfg<32>::G, NB = NP == 16 ? Cfg<16>::NB : Cfg<32>::NB;
  const int KS = (K + kStepRows - 1) / kStepRows;
  const int strips = M / 256;
  int ck = 1;
  for (int c : {2, 4, 8})
    if (strips * c <= sms && c <= KS) ck = c;
  const int nks = (KS + ck - 1) / ck;  // most K steps of any CTA
  const int xblocks = (nks + 3) / 4;
  const int xbytes = xblocks * NP * 128;
  const int need = (nks + kStageSteps - 1) / kStageSteps;
  int S = (kSmemBudget - 1024 - 256 - xbytes) / kStageBytes;
  S = std::min(std::min(S, kMaxStages), need);
  const int part = NP * 256 * 4;  // epilogue tile, reuses the stage ring
  if (S < 1) return false;
  if (S * kStageBytes < part) S = (part + kStageBytes - 1) / kStageBytes;
  pl->NP = NP;
  pl->Ck = ck;
  pl->S = S;
  pl->ctas = strips * ck;
  pl->xoff = S * kStageBytes;
  pl->xblocks = xblocks;
  pl->baroff = pl->xoff + xbytes;
  // + 4 KB of slack after the barriers; at least 116 KB: one CTA (and one TMEM
  // allocation) per SM, so two CTAs of one call never share an SM
  pl->smem = std::max(116 * 1024, 1024 + pl->baroff + (2 * kMaxStages + G * NB + G + 1) * 8 + 16 + 4096);
  const int cols = G * NB * 16 + 2 * G * NP;
  pl->tcols = cols <= 32 ? 32 : (cols <= 64 ? 64 : (cols <= 128 ? 128 : (cols <= 256 ? 256 : 512)));
  pl->ok = pl->tcols <= 256;
  return pl->ok;
}

template <int NP>
static int launch_np(const TcPlan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                     uint32_t* err, cudaStream_t st) {
  constexpr int G = Cfg<NP>::G, NB = Cfg<NP>::NB;
  auto kern = k_gemm_tc<NP, G, NB>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MB_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return MB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  CUtensorMap wmap, xmap;
  const uint64_t dims[3] = {kSB, static_cast<uint64_t>(M / 256), static_cast<uint64_t>(K)};
  const uint64_t strides[2] = {kSB, static_cast<uint64_t>(M / 256) * kSB};
  const uint32_t box[3] = {kSB, 1, kStageRows};
  if (!encode_tmap_3d_u8(&wmap, sb, dims, strides, box)) return MB_ERR_LAUNCH;
  // activations [N][K]: 64 x NP boxes, 128-byte rows swizzled (the tensor-core K-major layout)
  if (!encode_tmap_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                      static_cast<uint64_t>(K) * 2, 64, NP, CU_TENSOR_MAP_SWIZZLE_128B))
    return MB_ERR_LAUNCH;
  Params prm;
  prm.out = out;
  prm.err = err;
  prm.N = N;
  prm.K = K;
  prm.M = M;
  prm.KS = (K + kStepRows - 1) / kStepRows;
  prm.Ck = pl.Ck;
  prm.S = pl.S;
  prm.xoff = pl.xoff;
  prm.xblocks = pl.xblocks;
  prm.tcols = pl.tcols;
  prm.baroff = pl.baroff;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ctas);
  cfg.blockDim = dim3((2 + 4 * G) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = pl.Ck;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, wmap, xmap, prm) != cudaSuccess) return MB_ERR_LAUNCH;
  return launch_status();
}

int launch(const TcPlan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
           uint32_t* err, cudaStream_t st) {
  return pl.NP == 16 ? launch_np<16>(pl, act, sb, out, N, K, M, err, st)
                     : launch_np<32>(pl, act, sb, out, N, K, M, err, st);
}

}  // namespace tc
}  // namespace mb
