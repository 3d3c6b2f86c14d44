// Fused INT4 super-block batched GEMM for B200 (sm_100a):
//   out[N, M] (fp16) = act[N, K] (fp16) x dequant(sb)[K, M], fp32 accumulation.
//
// Replaces the reference's batched_gemm entry point (Metal batched_gemm_simdgroup /
// fused_batched_gemm_int4, antigravity-engine/src/shaders/batched_gemm.metal:74-169;
// CPU form `activations @ W`, batch_generator.py:290). The weight stream is the
// reference's 144-byte super-block format, read in place.
//
// Design (weight streaming, HBM bound):
//  * The M columns are cut into strips of WS = 256 (one super-block per row) or 128
//    columns. Each strip is handled by one thread-block cluster of Ck CTAs that
//    split its K rows; the grid (strips x Ck) is sized to one wave of the SMs. The
//    split-K partial sums are reduced on chip through distributed shared memory at
//    the end, so there is no global workspace, no atomics, and the result is
//    deterministic.
//  * One producer thread per CTA streams the strip's super-block rows with 3-D TMA
//    tile loads (cp.async.bulk.tensor, L2 evict-first) into a ring of shared-memory
//    stages guarded by mbarriers. The weights never depend on the previous kernel,
//    so the ring is filled before griddepcontrol.wait (programmatic dependent
//    launch). After it the consumer warps copy the CTA's activation slice (L2
//    resident) into shared memory with all loads of a round in flight.
//  * Consumer warps expand nibbles straight into mma.m16n8k16 A fragments in
//    registers: byte permute + magic-exponent fp16 conversion + one fp16 multiply by
//    the group scale, bit-exact with the reference dequant; the batch (padded to
//    8/16/32) is the MMA n dimension, fp32 accumulate.
//  * Reduction: the k-group warps park their partial tiles in the drained ring and sum
//    them in a fixed order into a send tile holding one block per owner CTA of the
//    cluster; one bulk shared-memory copy per peer (cp.async.bulk.shared::cluster)
//    moves each block, completion counted on the owner's mbarrier, and each owner adds
//    the Ck blocks of its columns in rank order.
//  * Shared-memory rows are laid out so the fragment loads are bank-conflict free:
//    full 144-byte super-block rows (WS = 256), or a 16-byte scale row plus a
//    nibble row padded to 80 / 96 bytes by the TMA box (WS = 128, M % 256 == 128).
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace mb {

constexpr int kSB = 144;        // bytes per super-block
constexpr int kSliceRows = 16;  // k rows per MMA slice
constexpr int kSPS = 8;         // slices per full stage (128 rows)
constexpr int kStageRows = kSPS * kSliceRows;
constexpr int kMaxStages = 8;
constexpr int kMaxCk = 8;
constexpr int kAhead = 3;  // weight stages in flight per CTA

// Shared-memory layout of one pipeline stage (128 rows of the CTA's strip).
//  WS = 256: full 144-byte super-block rows (scales then nibbles), row stride 144 B.
//  WS = 128 / 64: a 16-byte scale row per k row, then the strip's nibble bytes in a
//  row padded by the TMA box (80 / 48 bytes for one row phase, 96 / 32 bytes for two)
//  so that the fragment loads below hit 32 distinct banks. With P = 2 row phases
//  (M % 256 == 128) rows of each phase are stored together.
template <int WS, int P>
struct Layout {
  static_assert(WS == 256 || WS == 128, "strip width");
  static_assert(WS != 256 || P == 1, "a 256-wide strip needs M % 256 == 0");
  static_assert(P == 1 || P == 2, "row phases");
  static constexpr int kNibRow = (WS == 128) ? (P == 1 ? 80 : 96) : (P == 1 ? 48 : 32);
  static constexpr int kScRegion = kStageRows * 16;
  static constexpr int kStageBytes = (WS == 256) ? kStageRows * kSB : kStageRows * (16 + kNibRow);
  static constexpr int kRowsPerPhase = kStageRows / P;
  static __device__ __host__ constexpr int bytes(int n) {  // tx bytes of a stage with n slices
    return (WS == 256) ? n * kSliceRows * kSB : n * kSliceRows * (16 + kNibRow);
  }
  // byte offset of row k's scale chunk / first strip nibble byte within a stage
  static __device__ __forceinline__ constexpr int sc(int k) {
    return (WS == 256) ? k * kSB : ((k & (P - 1)) * kRowsPerPhase + k / P) * 16;
  }
  static __device__ __forceinline__ constexpr int nib(int k) {
    return (WS == 256) ? k * kSB + 16 : kScRegion + ((k & (P - 1)) * kRowsPerPhase + k / P) * kNibRow;
  }
};

struct GemmParams {
  uint16_t* out;        // [N, M] fp16
  const uint16_t* act;  // [N, K] fp16
  uint32_t* err;        // optional device error word (may be null)
  int N, K, M;
  int KS;               // k slices (ceil(K / 16))
  int Ck;               // CTAs per cluster = K split
  int S;                // stages in the ring
  int xchunks;          // 128-wide k chunks of the activation slice
  int xcstride;         // bytes per chunk in shared memory (N rows of kXRow bytes, 128-aligned)
  int sendoff;          // byte offset of the send tile [Ck][N][cwp] (reuses ring + activations)
  int baroff;           // byte offset of the mbarriers
  int recvoff;          // byte offset of the receive slots [Ck][N][cwp] (outside the ring)
};

// Activations in shared memory: chunks of 128 k values by N rows; a row takes 272
// bytes (128 values + 8 pad), so consecutive rows start 4 banks apart and the
// B-fragment loads are conflict free.
constexpr int kXChunk = 128;
constexpr int kXRow = 272;

struct WMaps {  // weight tensor maps: full-stage and 16-row boxes (scale / nibble rows)
  CUtensorMap full_a, full_b, slice_a, slice_b;
};

// Row stride (floats) of a k-group parking tile: WS columns with 2 pad floats after
// every MR-column run, and a stride of 4 (mod 16) between batch rows, so the float2
// stores of a warp's fragments hit distinct banks for MR = 32, 16 and 8.
template <int WS, int MR>
struct ParkRow {
  static constexpr int v = (WS + 2 * WS / MR - 4 + 15) / 16 * 16 + 4;
};

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
__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// One 16-row k slice for this thread's MR-column run.
// Thread (g4 = lane/4, t4 = lane%4) owns rows 2t4, 2t4+1, 2t4+8, 2t4+9 of the slice
// (the k positions of the m16n8k16 A fragment) and MR consecutive columns; m16 tile
// i of the warp maps fragment row g4 to column 2i and row g4+8 to column 2i+1 of the
// run, so each nibble byte feeds exactly one tile and the warp has MR/2 independent
// accumulator chains per batch tile. The weight operand is fp16((n - 8) * s): exact
// magic-exponent conversion of the nibble, then one rounding multiply by the group
// scale — bit-identical to the reference dequant.
//   stage, k0: stage base and the stage-local row 2t4 of this slice; nb: byte offset
//   of the run within a nibble row; ge / go: scale index for even / odd rows;
//   xrow: this lane's activation row (n = 8 nt + g4) at the slice's first k.
template <int NT, int WS, int P, int MR>
__device__ __forceinline__ void consume_slice(const uint8_t* stage, int k0, int nb, int ge, int go,
                                              const uint8_t* const (&xrow)[NT], const bool (&xok)[NT], int t4,
                                              float (&acc)[MR / 2][NT][4]) {
  using L = Layout<WS, P>;
  constexpr int NW = MR / 8;  // 32-bit nibble words per row
  // rows 2t4, 2t4+1, 2t4+8, 2t4+9 as constant offsets from row 2t4
  constexpr int dn1 = L::nib(1) - L::nib(0), dn8 = L::nib(8) - L::nib(0), dn9 = L::nib(9) - L::nib(0);
  constexpr int ds1 = L::sc(1) - L::sc(0), ds8 = L::sc(8) - L::sc(0), ds9 = L::sc(9) - L::sc(0);
  const uint8_t* pn = stage + L::nib(k0) + nb;
  const uint8_t* ps = stage + L::sc(k0);
  uint32_t w0[NW], w1[NW], w2[NW], w3[NW];
  lds_words<NW>(pn, w0);
  lds_words<NW>(pn + dn1, w1);
  lds_words<NW>(pn + dn8, w2);
  lds_words<NW>(pn + dn9, w3);
  const uint32_t s01 = lds_u16(ps + 2 * ge) | (lds_u16(ps + ds1 + 2 * go) << 16);
  const uint32_t s23 = lds_u16(ps + ds8 + 2 * ge) | (lds_u16(ps + ds9 + 2 * go) << 16);
  uint32_t bf[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    bf[nt][0] = xok[nt] ? lds_u32(xrow[nt] + 4 * t4) : 0u;
    bf[nt][1] = xok[nt] ? lds_u32(xrow[nt] + 16 + 4 * t4) : 0u;
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

template <int WS, int P>
__device__ __forceinline__ void issue_stage(const WMaps& maps, uint8_t* dst, uint64_t* bar, int k0, int n,
                                            const int (&ey)[P], const int (&ex)[P], uint64_t pol) {
  using L = Layout<WS, P>;
  mbar_expect_tx(bar, L::bytes(n));
  if constexpr (WS == 256) {
    if (n == kSPS) {
      tma_load_3d(dst, &maps.full_a, bar, 0, ey[0], k0, pol);
    } else {
      for (int j = 0; j < n; ++j)
        tma_load_3d(dst + j * kSliceRows * kSB, &maps.slice_a, bar, 0, ey[0], k0 + j * kSliceRows, pol);
    }
  } else {
    constexpr int rp = L::kRowsPerPhase;
#pragma unroll
    for (int r = 0; r < P; ++r) {
      uint8_t* sdst = dst + r * rp * 16;
      uint8_t* ndst = dst + L::kScRegion + r * rp * L::kNibRow;
      if (n == kSPS) {
        tma_load_3d(sdst, &maps.full_a, bar, 0, ey[r], k0 / P, pol);
        tma_load_3d(ndst, &maps.full_b, bar, ex[r], ey[r], k0 / P, pol);
      } else {
        constexpr int sp = kSliceRows / P;
        for (int j = 0; j < n; ++j) {
          tma_load_3d(sdst + j * sp * 16, &maps.slice_a, bar, 0, ey[r], (k0 + j * kSliceRows) / P, pol);
          tma_load_3d(ndst + j * sp * L::kNibRow, &maps.slice_b, bar, ex[r], ey[r], (k0 + j * kSliceRows) / P, pol);
        }
      }
    }
  }
}

__device__ __forceinline__ void store_half2(uint16_t* dst, float a, float b) {
  const __half2 x = __floats2half2_rn(a, b);
  *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(&x);
}

// Columns per thread run for (NT, WS): 32 / NT, at most WS / 8 (eight runs per warp).
template <int NT, int WS>
struct RunCols {
  static constexpr int v = (32 / NT < WS / 8) ? 32 / NT : WS / 8;
};

// NT: n-tiles of 8 batch rows (1, 2, 4); WS: strip width; P: row phases (1, 2);
// CW: consumer warps; MINB: CTAs per SM the plan wants resident -- 2 leaves room for
// the next call's CTA (launched early through PDL) to prefetch, 1 gives a CTA that
// has the SM to itself the registers for a deeper instruction schedule.
template <int NT, int WS, int P, int CW, int MINB>
__global__ void __launch_bounds__((CW + 1) * 32, MINB)
    k_gemm_int4(const __grid_constant__ WMaps maps, const GemmParams p) {
  using L = Layout<WS, P>;
  constexpr int MR = RunCols<NT, WS>::v;  // columns per thread run
  constexpr int kTiles = MR / 2;          // m16 tiles per warp
  constexpr int kCm = WS / (8 * MR);      // column parts per strip (one warp each)
  constexpr int kKG = CW / kCm;           // warps sharing a column part (k groups)
  static_assert(kCm * kKG == CW, "warp layout");
  constexpr int kRow = ParkRow<WS, MR>::v;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived from the shared array itself so that every access
  // below compiles to a shared-memory (not generic) load or store
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stages = smem;
  uint8_t* xs = stages + p.S * L::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kMaxStages;
  uint64_t* rbar = empty + kMaxStages;  // the peers' partial sums of this CTA's columns landed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = blockIdx.x / p.Ck;
  const int q = blockIdx.x - strip * p.Ck;  // == rank in the cluster (cluster dims = (Ck,1,1))
  const int sl0 = static_cast<int>((static_cast<long long>(q) * p.KS) / p.Ck);
  const int sl1 = static_cast<int>((static_cast<long long>(q + 1) * p.KS) / p.Ck);
  const int nst = (sl1 - sl0 + kSPS - 1) / kSPS;
  const int c0 = strip * WS;
  // CTA q of the cluster owns columns [q cw, min((q + 1) cw, WS)) of the strip:
  // ceil(WS / Ck) rounded up to even, so col / cw < Ck for every column. Partial sums
  // travel in blocks of N rows x cwp floats (a multiple of 16 bytes).
  const int cw = ((WS + p.Ck - 1) / p.Ck + 1) & ~1;
  const int cwp = (cw + 3) & ~3;
  const uint32_t blk = static_cast<uint32_t>(p.N * cwp * 4);
  // per row phase: super-block index within a period (y), first nibble byte of the
  // strip in that super-block (x) and the scale index of the strip's first column
  int ey[P], ex[P], grp[P];
#pragma unroll
  for (int r = 0; r < P; ++r) {
    const long long f = static_cast<long long>(r) * p.M + c0;
    ey[r] = static_cast<int>(f >> 8);
    const int e = static_cast<int>(f & 255);
    ex[r] = 16 + e / 2;
    grp[r] = e / 32;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, CW);
    }
    mbar_init(rbar, 1);
    fence_mbar_init();
    // this CTA's own arrival: the phase completes when the Ck - 1 peer blocks land
    if (p.Ck > 1) mbar_expect_tx(rbar, static_cast<uint32_t>(p.Ck - 1) * blk);
  }
  __syncthreads();
  if (p.Ck > 1) cluster_arrive();  // phase 0: the barriers above exist (awaited before any copy)
  pdl_launch_dependents();

  if (warp == CW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      // weights never depend on the previous grid: no griddepcontrol.wait here, so the
      // ring fills while the previous grid finishes
      const uint64_t pol = policy_evict_first();
      for (int st = 0; st < nst; ++st) {
        const int s = st % p.S;
        // at most kAhead stages in flight: the memory system then returns this CTA's
        // stages in order, so the first one lands early instead of with the last (with
        // kAhead <= S the slot of stage st - kAhead is not reused yet, so its parity is
        // unambiguous; with a shorter ring the empty wait below already implies it)
        if (st >= kAhead && kAhead <= p.S) {
          const int sa = st - kAhead;
          if (!mbar_wait(full + sa % p.S, (sa / p.S) & 1) && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
        }
        if (st >= p.S && !mbar_wait(empty + s, ((st / p.S) - 1) & 1) && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
        const int sl = sl0 + st * kSPS;
        issue_stage<WS, P>(maps, stages + s * L::kStageBytes, full + s, sl * kSliceRows, min(kSPS, sl1 - sl), ey, ex,
                           pol);
      }
    }
    __syncwarp();
    if (p.Ck > 1) {
      cluster_wait();
      cluster_arrive();
      cluster_wait();
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g4 = lane >> 2, t4 = lane & 3;
  const int mpart = warp % kCm, kg = warp / kCm;
  const int mcol = mpart * 8 * MR + g4 * MR;  // first column of this thread's run in the strip
  const int nb = mcol / 2;
  const int ge = grp[0] + mcol / 32, go = grp[P - 1] + mcol / 32;

  float acc[kTiles][NT][4];
#pragma unroll
  for (int i = 0; i < kTiles; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][nt][c] = 0.0f;
  bool xok[NT];
  const uint8_t* xbase[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nt * 8 + g4;
    xok[nt] = n < p.N;
    xbase[nt] = xs + (xok[nt] ? n : 0) * kXRow;
  }
  // Activation slice -> shared memory [chunk][n][kXRow] in 16-byte pieces: thread t
  // copies pieces t, t + T, t + 2T, ... of the [N][ppr] piece grid, kU loads in flight
  // per round, (n, pc) advanced incrementally (no division in the loop).
  pdl_wait();  // activations may come from the previous grid; all writes follow it
  {
    constexpr int T = CW * 32;
    constexpr int kU = 8;
    const int ppr = (sl1 - sl0) * kSliceRows / 8;  // pieces per row
    const int pieces = p.N * ppr;
    const int k0 = sl0 * kSliceRows;
    const int dn = T / ppr, dp = T - dn * ppr;
    int n = threadIdx.x / ppr, pc = threadIdx.x - n * ppr;
    for (int r0 = threadIdx.x; r0 < pieces; r0 += T * kU) {
      uint4 v[kU];
      int so[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        so[u] = -1;
        if (r0 + u * T < pieces) {
          const int k = k0 + pc * 8;
          if (k < p.K) v[u] = __ldg(reinterpret_cast<const uint4*>(p.act + static_cast<size_t>(n) * p.K + k));
          so[u] = (pc / (kXChunk / 8)) * p.xcstride + n * kXRow + (pc % (kXChunk / 8)) * 16;
        }
        pc += dp;
        n += dn;
        if (pc >= ppr) {
          pc -= ppr;
          ++n;
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (so[u] >= 0) *reinterpret_cast<uint4*>(xs + so[u]) = v[u];
    }
  }
  named_bar_sync(1, CW * 32);

  for (int st = 0; st < nst; ++st) {
    const int s = st % p.S;
    if (!mbar_wait(full + s, (st / p.S) & 1) && lane == 0 && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
    const uint8_t* stage = stages + s * L::kStageBytes;
    const int n = min(kSPS, sl1 - (sl0 + st * kSPS));
    for (int j = kg; j < n; j += kKG) {
      const int kx = (st * kSPS + j) * kSliceRows;  // k offset within the activation slice
      const int xo = (kx / kXChunk) * p.xcstride + (kx % kXChunk) * 2;
      const uint8_t* xr[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xr[nt] = xbase[nt] + xo;
      consume_slice<NT, WS, P, MR>(stage, j * kSliceRows + 2 * t4, nb, ge, go, xr, xok, t4, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
  }

  // ---- k groups -> one partial tile per CTA ----
  // Park the partial sums of the batch rows n < N in [kKG][N][kRow] (the ring and the
  // activations are drained): thread (g4, t4) holds rows 8 nt + 2 t4 + (c & 1) of
  // columns mcol + 2 i + (c >> 1).
  named_bar_sync(1, CW * 32);
  float* park = reinterpret_cast<float*>(smem);
  {
    float* rbase = park + (kg * p.N + 2 * t4) * kRow + mcol + 2 * (mcol / MR);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        if (nt * 8 + 2 * t4 + r < p.N) {
          float* row = rbase + (nt * 8 + r) * kRow;
#pragma unroll
          for (int i = 0; i < kTiles; ++i)
            *reinterpret_cast<float2*>(row + 2 * i) = make_float2(acc[i][nt][r], acc[i][nt][r + 2]);
        }
      }
  }
  named_bar_sync(1, CW * 32);
  // sum the k groups in order; Ck == 1: that is the result, else it goes to the send
  // tile, one block of N x cwp floats per owner CTA. Thread t keeps one column pair and
  // walks the batch rows (WS / 2 divides the consumer thread count).
  float* send = reinterpret_cast<float*>(smem + p.sendoff);
  {
    constexpr int kPairs = WS / 2, kDn = CW * 32 / kPairs;
    static_assert(CW * 32 % kPairs == 0, "column pairs per pass");
    const int col = 2 * (threadIdx.x % kPairs);
    const int o = col / cw, lc = col - o * cw;
    const float* src = park + col + 2 * (col / MR);
    for (int n = threadIdx.x / kPairs; n < p.N; n += kDn) {
      float lo = 0.0f, hi = 0.0f;
#pragma unroll
      for (int g = 0; g < kKG; ++g) {
        const float2 v = *reinterpret_cast<const float2*>(src + (g * p.N + n) * kRow);
        lo += v.x;
        hi += v.y;
      }
      if (p.Ck == 1)
        store_half2(p.out + static_cast<size_t>(n) * p.M + c0 + col, lo, hi);
      else
        *reinterpret_cast<float2*>(send + (o * p.N + n) * cwp + lc) = make_float2(lo, hi);
    }
  }
  if (p.Ck == 1) return;

  // ---- partial tiles -> owner CTAs: one bulk copy per peer, completion on its rbar ----
  fence_proxy_async_smem();
  named_bar_sync(1, CW * 32);
  cluster_wait();  // phase 0: every peer's rbar is initialised
  const float* recv = reinterpret_cast<const float*>(smem + p.recvoff);  // [Ck][N][cwp], slot = sender
  if (threadIdx.x == 0) {
    for (int o = 0; o < p.Ck; ++o) {
      if (o == q) continue;
      bulk_copy_to_peer(mapa_shared(smem_u32(recv) + static_cast<uint32_t>(q) * blk, static_cast<uint32_t>(o)),
                        send + o * p.N * cwp, blk, mapa_shared(smem_u32(rbar), static_cast<uint32_t>(o)));
    }
  }
  if (!mbar_wait(rbar, 0) && lane == 0 && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
  const int mine = min(cw, WS - q * cw);  // columns this CTA owns (may be <= 0)
  if (mine > 0) {
    // thread t: column pair i, batch row n of item t of the [N][mine / 2] grid, advanced
    // by the thread count without a division in the loop
    const int mp = mine / 2, T = CW * 32;
    const int dn = T / mp, di = T - dn * mp;
    int n = threadIdx.x / mp, i = threadIdx.x - n * mp;
    while (n < p.N) {
      const int lc = 2 * i;
      float lo = 0.0f, hi = 0.0f;
      for (int c = 0; c < p.Ck; ++c) {
        const float* src = (c == q) ? send + (q * p.N + n) * cwp : recv + (c * p.N + n) * cwp;
        const float2 v = *reinterpret_cast<const float2*>(src + lc);
        lo += v.x;
        hi += v.y;
      }
      store_half2(p.out + static_cast<size_t>(n) * p.M + c0 + q * cw + lc, lo, hi);
      n += dn;
      i += di;
      if (i >= mp) {
        i -= mp;
        ++n;
      }
    }
  }
  // phase 1: every block addressed to this CTA has landed (a relaxed arrival: a release
  // would first wait for this thread's output stores, which the phase does not need)
  cluster_arrive_relaxed();
  cluster_wait();  // phase 1: no peer still reads this CTA's send tile
}

// ---------------------------------------------------------------------------
// Generic path (any M with K*M % 256 == 0, any K): one thread per output column,
// flat super-block indexing as in fused_batched_gemm_int4 (batched_gemm.metal:146-155),
// activations staged in shared memory. Correct for every shape; the TMA path above
// is the fast one.
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(128) k_gemm_generic(const uint16_t* __restrict__ act, const uint8_t* __restrict__ sb,
                                                      uint16_t* __restrict__ out, int N, int K, int M) {
  constexpr int KC = 64;
  __shared__ float xsm[NB][KC];
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  float acc[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += KC) {
    __syncthreads();
    for (int t = threadIdx.x; t < NB * KC; t += blockDim.x) {
      const int n = t / KC, kk = t % KC;
      xsm[n][kk] = (n < N && k0 + kk < K) ? __half2float(__ushort_as_half(act[static_cast<size_t>(n) * K + k0 + kk]))
                                          : 0.0f;
    }
    __syncthreads();
    if (m < M) {
      const int kend = min(KC, K - k0);
      for (int kk = 0; kk < kend; ++kk) {
        const long long flat = static_cast<long long>(k0 + kk) * M + m;
        const uint8_t* b = sb + (flat >> 8) * kSB;
        const int e = static_cast<int>(flat & 255);
        const int byte = __ldg(b + 16 + (e >> 1));
        const int qv = ((e & 1) ? (byte >> 4) : (byte & 15)) - 8;
        const __half s = __ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(b) + (e >> 5)));
        const float w = __half2float(__hmul(__int2half_rn(qv), s));
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(xsm[n][kk], w, acc[n]);
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
struct Plan {
  int ws = 0, P = 1, Ck = 1, nt = 1, S = 0, smem = 0, ctas = 0;
  int xchunks = 0, xcstride = 0, xbytes = 0, sendoff = 0, baroff = 0, recvoff = 0;
  bool fast = false;
  bool solo = false;  // one CTA per SM
};

static constexpr int kCW = 8;                   // consumer warps per CTA
static constexpr int kSmemBudget = 112 * 1024;  // half an SM: room for the next call's CTA

static int stage_bytes_of(int ws, int P) {
  if (ws == 256) return Layout<256, 1>::kStageBytes;
  return P == 1 ? Layout<128, 1>::kStageBytes : Layout<128, 2>::kStageBytes;
}

static inline int round_up(int x, int a) { return (x + a - 1) / a * a; }

// bytes of the k-group parking tile [kKG][N][kRow] of the final reduction
static int park_bytes(int nt, int ws, int N) {
  const int mr = std::min(32 / nt, ws / 8);
  const int kg = kCW / (ws / (8 * mr));
  const int row = (ws + 2 * ws / mr - 4 + 15) / 16 * 16 + 4;  // ParkRow<ws, mr>
  return kg * N * row * 4;
}

// bytes of one owner block of partial sums (N rows x cwp floats), as in the kernel
static int owner_block_bytes(int ws, int ck, int N) {
  const int cw = ((ws + ck - 1) / ck + 1) & ~1;
  return N * ((cw + 3) & ~3) * 4;
}

// The complete launch plan of one (strip width, cluster size) candidate: ring depth,
// shared-memory layout and residency. pl.fast is false if it does not fit.
static Plan make_plan(int N, int KS, int P, int ws, int ck) {
  Plan pl;
  pl.nt = N <= 8 ? 1 : (N <= 16 ? 2 : 4);
  pl.P = P;
  pl.ws = ws;
  pl.Ck = ck;
  pl.xcstride = round_up(N * kXRow, 128);
  const int KSc = (KS + ck - 1) / ck;
  pl.xbytes = (KSc * kSliceRows + kXChunk - 1) / kXChunk * pl.xcstride;
  pl.xchunks = pl.xbytes / pl.xcstride;
  const int sb = stage_bytes_of(ws, P);
  if (pl.xbytes + 2 * sb + 2048 > 220 * 1024) return pl;  // a large activation slice makes the CTA solo
  const int need = (KSc + kSPS - 1) / kSPS;  // stages that hold the CTA's whole slice
  // A CTA with a large share of the weights computes for long: one CTA per SM (at least
  // 116 KB), since two CTAs of one call on an SM take twice as long and hold back the
  // whole call. A small share is dominated by start-up latency: leave room for the next
  // call's CTA to start early (programmatic dependent launch) and prefetch.
  pl.solo = static_cast<long long>(ws) * KSc * kSliceRows >= 64 * 1024;
  const int blk = owner_block_bytes(ws, ck, N);
  const int recvbytes = ck > 1 ? ck * blk : 0;
  if (pl.xbytes + 2 * sb + 2048 > kSmemBudget) pl.solo = true;
  const int budget = pl.solo ? std::max(116 * 1024, pl.xbytes + recvbytes + 2048 + 2 * sb) : kSmemBudget;
  int S = (budget - 2048 - pl.xbytes - recvbytes) / sb;
  S = std::max(2, std::min(std::min(S, kMaxStages), need));
  // the parking tile and the send tile live in the drained ring + activation region
  pl.sendoff = round_up(park_bytes(pl.nt, ws, N), 16);
  const int rb = pl.sendoff + (ck > 1 ? ck * blk : 0);
  while (S * sb + pl.xbytes < rb && S < kMaxStages) ++S;
  pl.S = S;
  pl.baroff = round_up(std::max(S * sb + pl.xbytes, rb), 16);
  pl.recvoff = pl.baroff + (2 * kMaxStages + 2) * 8;  // full, empty, rbar (+ pad)
  pl.smem = 1024 + pl.recvoff + recvbytes;
  if (pl.smem > 113 * 1024) pl.solo = true;  // two CTAs do not fit an SM anyway: take the registers
  if (pl.solo) pl.smem = std::max(pl.smem, 116 * 1024);
  pl.fast = pl.smem <= 227 * 1024;
  return pl;
}

template <int NT, int WS, int P, int MINB>
static int max_clusters_q(int ck, int smem) {
  auto kern = k_gemm_int4<NT, WS, P, kCW, MINB>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ck * 16);
  cfg.blockDim = dim3((kCW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = ck;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return n;
}

// How many clusters of a plan the GPU holds at once (cudaOccupancyMaxActiveClusters on
// the plan's own kernel). Without a device: the counts measured on B200 for one CTA per
// SM (clusters of 7 and 8 fit only 15 times: a GPC holds two), scaled to the SM count.
static int max_clusters(const Plan& pl, int sms) {
  int n = -1;
  const int minb = pl.solo ? 1 : 2;
#define MB_Q(NT_, WS_, P_)                                                                  \
  if (pl.nt == NT_ && pl.ws == WS_ && pl.P == P_)                                           \
    n = minb == 1 ? max_clusters_q<NT_, WS_, P_, 1>(pl.Ck, pl.smem) : max_clusters_q<NT_, WS_, P_, 2>(pl.Ck, pl.smem);
  MB_Q(1, 256, 1) MB_Q(1, 128, 1) MB_Q(1, 128, 2) MB_Q(2, 256, 1) MB_Q(2, 128, 1) MB_Q(2, 128, 2)
  MB_Q(4, 256, 1) MB_Q(4, 128, 1) MB_Q(4, 128, 2)
#undef MB_Q
  if (n > 0) return n;
  static const int solo148[kMaxCk + 1] = {0, 148, 74, 45, 33, 26, 22, 15, 15};
  const int base = solo148[pl.Ck] * sms / 148;
  return pl.solo ? base : 2 * base;
}

// Estimated time (ns) of one call under a plan, fitted to measurements on B200:
//  * ~3.75 us of fixed cost (launch hand-off, activation copy, first weight stage,
//    cross-CTA reduction);
//  * the dequant loop at ~34 / 23 / 15 weights per cycle per SM for thread runs of
//    32 / 16 / 8 columns (MR), ~1.85 GHz under load;
//  * the weight stream at ~6.5 TB/s as a floor;
//  * a cluster grid larger than the clusters the GPU holds at once runs in two waves.
static double plan_cost(const Plan& pl, int N, int K, int M, int KS, int sms) {
  const int KSc = (KS + pl.Ck - 1) / pl.Ck;
  const double w_cta = static_cast<double>(pl.ws) * KSc * kSliceRows;
  const int mr = std::min(32 / pl.nt, pl.ws / 8);
  const double rate = mr >= 32 ? 34.0 : (mr >= 16 ? 23.0 : 15.0);
  double t = 3750.0 + w_cta / rate / 1.85;
  const double bytes = static_cast<double>(K) * M * kSB / 256 + 2.0 * N * (K + M);
  t = std::max(t, 1500.0 + bytes / 6500.0);  // 6.5 TB/s = 6500 bytes per ns
  if (pl.Ck > 1 && pl.ctas / pl.Ck > max_clusters(pl, sms)) t += 4000.0;
  return t;
}

// Picks the strip width and K split (cluster size) with the lowest estimated time;
// ties go to the wider strip and fewer CTAs per cluster.
static Plan plan_gemm_uncached(int N, int K, int M, int sms) {
  Plan best;
  best.nt = N <= 8 ? 1 : (N <= 16 ? 2 : 4);
  if (K % 8 != 0 || M % 128 != 0) return best;
  const int P = (M % 256 == 0) ? 1 : ((M % 128 == 0) ? 2 : 0);
  if (P == 0) return best;
  const int KS = (K + kSliceRows - 1) / kSliceRows;
  double best_t = 0.0;
  for (int ws : {256, 128}) {
    if (ws == 256 && P != 1) continue;
    const int strips = M / ws;
    for (int ck = 1; ck <= kMaxCk && ck <= KS; ++ck) {
      const long long ctas = static_cast<long long>(strips) * ck;
      if (ck > 1 && ctas > sms) break;  // a cluster grid must fit one wave
      Plan pl = make_plan(N, KS, P, ws, ck);
      if (!pl.fast) continue;
      pl.ctas = static_cast<int>(ctas);
      const double t = plan_cost(pl, N, K, M, KS, sms);
      if (!best.fast || t < best_t - 1e-6) {
        best = pl;
        best_t = t;
      }
    }
  }
  return best;
}

// Plans are cached per (device, N, K, M): the capacity query is not free and a decode
// loop repeats a handful of shapes.
static Plan plan_gemm(int N, int K, int M, int sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    dev = -1;
  }
  const uint64_t key = (static_cast<uint64_t>(static_cast<uint32_t>(dev) & 0xFF) << 56) ^
                       (static_cast<uint64_t>(N) << 48) ^ (static_cast<uint64_t>(static_cast<uint32_t>(K)) << 24) ^
                       static_cast<uint64_t>(static_cast<uint32_t>(M));
  static std::mutex mu;
  static std::unordered_map<uint64_t, Plan> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const Plan pl = plan_gemm_uncached(N, K, M, sms);
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, pl);
  return pl;
}

// Tensor maps of a weight stream: 3-D view [144 bytes][super-blocks per period]
// [periods of P rows], full-stage and 16-row boxes. Encoding costs a few microseconds
// of host time per launch, so maps are cached per (address, K, M, strip, phases): a
// decode loop streams the same weight tensors every step. A map depends only on these
// values, so a cached entry stays valid for any tensor at that address and shape.
template <int WS, int P>
static bool weight_maps(const uint8_t* sb, int K, int M, WMaps* maps) {
  using L = Layout<WS, P>;
  struct Key {
    const uint8_t* sb;
    int K, M;
    bool operator==(const Key& o) const { return sb == o.sb && K == o.K && M == o.M; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.sb) ^ (static_cast<size_t>(k.K) * 0x9E3779B97F4A7C15ull) ^
             (static_cast<size_t>(k.M) << 1);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, WMaps, Hash> cache;
  const Key key{sb, K, M};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *maps = it->second;
      return true;
    }
  }
  const uint64_t sbp = static_cast<uint64_t>(P) * M / 256;
  const uint64_t dims[3] = {kSB, sbp, static_cast<uint64_t>(K / P)};
  const uint64_t strides[2] = {kSB, sbp * kSB};
  bool ok;
  if (WS == 256) {
    const uint32_t bf[3] = {kSB, 1, kStageRows}, bs[3] = {kSB, 1, kSliceRows};
    ok = encode_tmap_3d_u8(&maps->full_a, sb, dims, strides, bf) &&
         encode_tmap_3d_u8(&maps->slice_a, sb, dims, strides, bs);
    maps->full_b = maps->full_a;
    maps->slice_b = maps->slice_a;
  } else {
    const uint32_t sf[3] = {16, 1, kStageRows / P}, ss[3] = {16, 1, kSliceRows / P};
    const uint32_t nf[3] = {L::kNibRow, 1, kStageRows / P}, ns[3] = {L::kNibRow, 1, kSliceRows / P};
    ok = encode_tmap_3d_u8(&maps->full_a, sb, dims, strides, sf) &&
         encode_tmap_3d_u8(&maps->slice_a, sb, dims, strides, ss) &&
         encode_tmap_3d_u8(&maps->full_b, sb, dims, strides, nf) &&
         encode_tmap_3d_u8(&maps->slice_b, sb, dims, strides, ns);
  }
  if (!ok) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 4096) cache.clear();
  cache.emplace(key, *maps);
  return true;
}

template <int NT, int WS, int P, int MINB>
static int launch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                       uint32_t* err, cudaStream_t st) {
  auto kern = k_gemm_int4<NT, WS, P, kCW, MINB>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MB_ERR_LAUNCH;
  if (!attr_set[dev]) {
    // full shared-memory carveout, so two ~112 KB CTAs (this call and the next) fit an SM
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return MB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  WMaps maps;
  if (!weight_maps<WS, P>(sb, K, M, &maps)) return MB_ERR_LAUNCH;
  GemmParams prm;
  prm.out = out;
  prm.act = act;
  prm.err = err;
  prm.N = N;
  prm.K = K;
  prm.M = M;
  prm.KS = (K + kSliceRows - 1) / kSliceRows;
  prm.Ck = pl.Ck;
  prm.S = pl.S;
  prm.xchunks = pl.xchunks;
  prm.xcstride = pl.xcstride;
  prm.sendoff = pl.sendoff;
  prm.baroff = pl.baroff;
  prm.recvoff = pl.recvoff;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M / WS) * pl.Ck);
  cfg.blockDim = dim3((kCW + 1) * 32);
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
  if (cudaLaunchKernelEx(&cfg, kern, maps, prm) != cudaSuccess) return MB_ERR_LAUNCH;
  return launch_status();
}

template <int NT, int MINB>
static int dispatch_fast_b(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                           uint32_t* err, cudaStream_t st) {
  if (pl.ws == 256) return launch_fast<NT, 256, 1, MINB>(pl, act, sb, out, N, K, M, err, st);
  if (pl.ws == 128)
    return pl.P == 1 ? launch_fast<NT, 128, 1, MINB>(pl, act, sb, out, N, K, M, err, st)
                     : launch_fast<NT, 128, 2, MINB>(pl, act, sb, out, N, K, M, err, st);
  return MB_ERR_UNSUPPORTED;
}

template <int NT>
static int dispatch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                         uint32_t* err, cudaStream_t st) {
  return pl.solo ? dispatch_fast_b<NT, 1>(pl, act, sb, out, N, K, M, err, st)
                 : dispatch_fast_b<NT, 2>(pl, act, sb, out, N, K, M, err, st);
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

// One launch over up to 32 batch rows: the cluster kernel, else the generic one.
static int gemm_rows(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, uint32_t* err,
                     cudaStream_t st) {
  if (aligned(act, 16) && aligned(sb, 16) && aligned(out, 4)) {
    const Plan pl = plan_gemm(N, K, M, sm_count());
    if (pl.fast) {
      if (pl.nt == 1) return dispatch_fast<1>(pl, act, sb, out, N, K, M, err, st);
      if (pl.nt == 2) return dispatch_fast<2>(pl, act, sb, out, N, K, M, err, st);
      return dispatch_fast<4>(pl, act, sb, out, N, K, M, err, st);
    }
  }
  return launch_generic(act, sb, out, N, K, M, st);
}

static int gemm_all(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                    uint32_t* dev_err, void* stream) {
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  if (!act || !sb || !out) return MB_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < N; r0 += 32) {
    const int nb = std::min(32, N - r0);
    const int rc = gemm_rows(act + static_cast<size_t>(r0) * K, sb, out + static_cast<size_t>(r0) * M, nb, K, M,
                             dev_err, st);
    if (rc != MB_OK) return rc;
  }
  return MB_OK;
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_int4_gemm(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                     uint32_t* dev_err, void* stream) {
  return gemm_all(act, sb, out, N, K, M, dev_err, stream);
}

int32_t mb_int4_gemm_host(const uint16_t* act_host, const uint8_t* sb, uint16_t* out_host, int32_t N, int32_t K,
                          int32_t M, uint16_t* act_dev, uint16_t* out_dev, uint32_t* dev_err, void* stream) {
  if (!act_host || !sb || !out_host || !act_dev || !out_dev) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t in_bytes = static_cast<size_t>(N) * K * 2, out_bytes = static_cast<size_t>(N) * M * 2;
  if (cudaMemcpyAsync(act_dev, act_host, in_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  const int32_t rc = gemm_all(act_dev, sb, out_dev, N, K, M, dev_err, stream);
  if (rc != MB_OK) return rc;
  if (cudaMemcpyAsync(out_host, out_dev, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

int32_t mb_int4_gemm_plan(int32_t N, int32_t K, int32_t M, int32_t* info) {
  if (!info) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1) return MB_ERR_ARGS;
  const Plan pl = plan_gemm(std::min(N, 32), K, M, sm_count());
  info[0] = pl.fast ? 1 : 0;
  info[1] = pl.ws;
  info[2] = pl.Ck;
  info[3] = pl.fast ? pl.ctas : (M + 127) / 128;
  info[4] = pl.S;
  info[5] = pl.smem;
  info[6] = pl.P;
  info[7] = pl.nt;
  return MB_OK;
}

}  // extern "C"
