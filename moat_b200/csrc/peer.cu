// Tensor-parallel exchanges of the decode step over NVLink peer memory (B200, sm_100a).
//
// A row-parallel projection (o_proj, down) leaves on every rank a partial product
// [N, D]; the next operation is the residual add and RMSNorm of the sum over ranks
// (transformer.py:148-158 on one device). A column-split lm_head leaves per rank the
// logits of its vocabulary range; the greedy choice is the argmax over all of them
// (batch_generator.py:203-206, 224-227). Instead of a library all-reduce followed by
// separate kernels, each exchange here is ONE kernel per rank that stores its rows
// straight into the other ranks' exchange buffers (plain peer stores over NVLink, no
// multicast), publishes them with a release flag, waits (bounded) for every rank's
// rows and finishes the operation locally:
//   k_peer_add_rmsnorm : sum the N x D partials in rank order in fp32, round to fp16
//                        (the all-reduced projection), x += it, h = RMSNorm(x) * w;
//   k_peer_argmax      : best (value, column) key of this rank's logits row, exchanged,
//                        integer max over ranks -> token id.
// Every rank sums the same values in the same order, so the residual streams stay
// bit-identical across ranks.
//
// Exchange buffer (one per rank, cudaMalloc + CUDA IPC, zeroed at creation):
//   [0, 2048)            flags of channel 0 (add_rmsnorm): uint32 [kMaxRows][kMaxRanks]
//   [2048, 4096)         flags of channel 1 (argmax)
//   [4096, 12288)        channel 1 keys: int64 [2 parities][kMaxRanks][kMaxRows]
//   [16384, ...)         channel 0 rows: fp16 [2 parities][kMaxRanks][slot_elems]
// flags[n][q] at rank r holds the last epoch in which rank q delivered row n to r.
// Epoch e (1, 2, ...) of a channel writes parity e & 1; a rank can only reach epoch
// e + 2 after every rank has finished epoch e + 1, hence finished reading epoch e's
// parity, so two parities never race. The epoch counter of each channel lives in a
// small local state array (not shared) and is advanced by the last CTA of each call,
// which keeps a captured CUDA graph replayable.
//
// Both kernels are chained with programmatic dependent launch: each waits for the
// previous kernel to finish before it reads anything (griddepcontrol.wait), then lets
// the next kernel start its prologue, which itself waits for this grid before it reads
// x, h or ids; all CTAs of an exchange are resident before a dependent grid launches.
//
// Every wait is bounded by the global timer: on expiry the kernel sets
// MB_DEVERR_TIMEOUT in dev_err and carries on (its outputs are then undefined).
// Ranks must run on distinct GPUs: two ranks' kernels waiting on each other are never
// both resident on one GPU; the host layer checks the device UUIDs before the buffers
// are exchanged.
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"

namespace mb {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxRows = 64;
constexpr int kPeerBlock = 256;
constexpr size_t kPeerFlagBytes = sizeof(uint32_t) * kPeerMaxRows * kPeerMaxRanks;  // 2048 per channel
constexpr size_t kPeerKeyOff = 2 * kPeerFlagBytes;
constexpr size_t kPeerRowOff = 16384;
static_assert(kPeerKeyOff + 2 * kPeerMaxRanks * kPeerMaxRows * sizeof(int64_t) <= kPeerRowOff, "layout");

struct PeerSet {
  uint8_t* buf[kPeerMaxRanks];  // every rank's exchange buffer as mapped in this process (own included)
  int world;
  int rank;
  int64_t slot_elems;  // fp16 elements of one channel-0 slot (>= N * D)
  int64_t timeout_ns;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t* peer_flag(uint8_t* buf, int channel, int row, int src) {
  return reinterpret_cast<uint32_t*>(buf + channel * kPeerFlagBytes) + row * kPeerMaxRanks + src;
}

// Publish this CTA's stores (all threads, before the barrier) to every rank, then wait
// for every rank's row `row` of epoch `epoch`. Threads q < world each own one rank.
__device__ __forceinline__ void peer_signal_and_wait(const PeerSet& ps, int channel, int row, uint32_t epoch,
                                                     uint32_t* err) {
  __syncthreads();
  const int q = threadIdx.x;
  if (q < ps.world) {
    __threadfence_system();
    st_release_sys(peer_flag(ps.buf[q], channel, row, ps.rank), epoch);
    const uint32_t* f = peer_flag(ps.buf[ps.rank], channel, row, q);
    const uint64_t t0 = global_ns();
    while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      if (global_ns() - t0 > static_cast<uint64_t>(ps.timeout_ns)) {
        if (err) atomicOr(err, MB_DEVERR_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// The last CTA of a call advances the channel's epoch (read by the next call).
__device__ __forceinline__ void peer_finish(uint32_t* state, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(state + 1, 1u) == gridDim.x - 1) {
      state[1] = 0;
      state[0] = epoch;
      __threadfence();
    }
  }
}

__device__ __forceinline__ float block_sum_fixed(float v, float* part) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kPeerBlock / 32; ++i) tot += part[i];  // fixed order: deterministic
  return tot;
}

// One CTA per row n. state = {epoch, arrivals} of channel 0.
__global__ void __launch_bounds__(kPeerBlock) k_peer_add_rmsnorm(PeerSet ps, const uint16_t* __restrict__ partial,
                                                                 float* __restrict__ x, const float* __restrict__ w,
                                                                 int D, float eps, uint16_t* __restrict__ h,
                                                                 uint32_t* state, uint32_t* err) {
  extern __shared__ float delta[];  // [D]: the all-reduced row, fp16-rounded, as float
  __shared__ float part[kPeerBlock / 32];
  pdl_wait();               // the partial and the epoch state come from earlier kernels
  pdl_launch_dependents();  // the next kernel's prologue may overlap; it waits for this grid before reading x, h
  const int n = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(state) + 1u;
  const int par = epoch & 1u;
  const int vecs = D / 8;  // 16-byte vectors per row
  auto slot = [&](uint8_t* buf, int src) {
    return reinterpret_cast<uint4*>(buf + kPeerRowOff) +
           ((static_cast<int64_t>(par) * kPeerMaxRanks + src) * ps.slot_elems + static_cast<int64_t>(n) * D) / 8;
  };
  // 1. this rank's row n into slot [par][rank] of every rank (its own buffer included)
  const uint4* src = reinterpret_cast<const uint4*>(partial + static_cast<int64_t>(n) * D);
  for (int i = threadIdx.x; i < vecs; i += kPeerBlock) {
    const uint4 v = src[i];
    for (int q = 0; q < ps.world; ++q) slot(ps.buf[q], ps.rank)[i] = v;
  }
  peer_signal_and_wait(ps, 0, n, epoch, err);
  // 2. sum the ranks' rows in rank order (fp32), one fp16 rounding
  for (int i = threadIdx.x; i < vecs; i += kPeerBlock) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    for (int q = 0; q < ps.world; ++q) {
      const uint4 v = __ldcg(slot(ps.buf[ps.rank], q) + i);
      const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(hv[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) delta[8 * i + j] = __half2float(__float2half_rn(acc[j]));
  }
  __syncthreads();
  // 3. residual add and RMSNorm, element order as k_add_rmsnorm
  float* xr = x + static_cast<int64_t>(n) * D;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < D; c += kPeerBlock) {
    const float v = xr[c] + delta[c];
    xr[c] = v;
    ss = fmaf(v, v, ss);
  }
  const float inv = rsqrtf(block_sum_fixed(ss, part) / static_cast<float>(D) + eps);
  for (int c = threadIdx.x; c < D; c += kPeerBlock)
    h[static_cast<int64_t>(n) * D + c] = __half_as_ushort(__float2half_rn(xr[c] * inv * w[c]));
  peer_finish(state, epoch);
}

// One CTA per row n: key of this rank's best logit, exchanged, max over ranks -> ids[n].
// state = {epoch, arrivals} of channel 1.
constexpr int kPeerArgBlock = 1024;

__global__ void __launch_bounds__(kPeerArgBlock) k_peer_argmax(PeerSet ps, const uint16_t* __restrict__ logits, int V,
                                                               int col0, int32_t* __restrict__ ids, uint32_t* state,
                                                               uint32_t* err) {
  __shared__ unsigned long long best_w[kPeerArgBlock / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(state) + 1u;
  const int par = epoch & 1u;
  unsigned long long best =
      thread_best_key(logits + static_cast<int64_t>(n) * V, V, col0, threadIdx.x, kPeerArgBlock);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) best_w[threadIdx.x >> 5] = best;
  __syncthreads();
  auto key_slot = [&](uint8_t* buf, int src) {
    return reinterpret_cast<unsigned long long*>(buf + kPeerKeyOff) + (par * kPeerMaxRanks + src) * kPeerMaxRows + n;
  };
  if (threadIdx.x < ps.world) {
    unsigned long long b = best_w[0];
    for (int i = 1; i < kPeerArgBlock / 32; ++i) b = best_w[i] > b ? best_w[i] : b;
    *key_slot(ps.buf[threadIdx.x], ps.rank) = b;
  }
  peer_signal_and_wait(ps, 1, n, epoch, err);
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int q = 0; q < ps.world; ++q) {
      const unsigned long long k = __ldcg(key_slot(ps.buf[ps.rank], q));
      b = k > b ? k : b;
    }
    ids[n] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(b & 0xFFFFFFFFull));
  }
  peer_finish(state, epoch);
}

static bool make_peer_set(void* const* bufs, int world, int rank, int64_t slot_elems, int64_t timeout_ns,
                          PeerSet* ps) {
  if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world || slot_elems < 8 || slot_elems % 8 != 0 ||
      timeout_ns <= 0)
    return false;
  for (int q = 0; q < kPeerMaxRanks; ++q) {
    ps->buf[q] = q < world ? static_cast<uint8_t*>(bufs[q]) : nullptr;
    if (q < world && (!bufs[q] || !aligned(bufs[q], 256))) return false;
  }
  ps->world = world;
  ps->rank = rank;
  ps->slot_elems = slot_elems;
  ps->timeout_ns = timeout_ns;
  return true;
}

}  // namespace mb

using namespace mb;

extern "C" {

size_t mb_peer_buffer_bytes(int32_t max_rows, int32_t D) {
  if (max_rows < 1 || max_rows > kPeerMaxRows || D < 8 || D % 8 != 0) return 0;
  const size_t slot = static_cast<size_t>(max_rows) * D;
  return kPeerRowOff + 2 * kPeerMaxRanks * slot * sizeof(uint16_t);
}

int32_t mb_ipc_alloc(size_t bytes, void** ptr, uint8_t* handle) {
  if (!ptr || !handle) return MB_ERR_NULL;
  if (bytes == 0) return MB_ERR_ARGS;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    return MB_ERR_LAUNCH;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MB_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MB_OK;
}

int32_t mb_ipc_open(const uint8_t* handle, void** ptr) {
  if (!handle || !ptr) return MB_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  *ptr = p;
  return MB_OK;
}

int32_t mb_ipc_close(void* ptr) {
  if (!ptr) return MB_ERR_NULL;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

int32_t mb_ipc_free(void* ptr) {
  if (!ptr) return MB_ERR_NULL;
  if (cudaFree(ptr) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

int32_t mb_peer_add_rmsnorm(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                            const uint16_t* partial, float* x, const float* w, int32_t N, int32_t D, float eps,
                            uint16_t* h, uint32_t* state, uint32_t* dev_err, void* stream) {
  if (!bufs || !partial || !x || !w || !h || !state) return MB_ERR_NULL;
  if (N < 1 || N > kPeerMaxRows || D < 8 || D % 8 != 0 || static_cast<int64_t>(N) * D > slot_elems ||
      D > 16384)
    return MB_ERR_ARGS;
  if (!aligned(partial, 16)) return MB_ERR_ALIGN;
  PeerSet ps;
  if (!make_peer_set(bufs, world, rank, slot_elems, timeout_ns, &ps)) return MB_ERR_ARGS;
  const size_t smem = static_cast<size_t>(D) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k_peer_add_rmsnorm, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess)
    return MB_ERR_LAUNCH;
  return launch_with_pdl(k_peer_add_rmsnorm, dim3(N), dim3(kPeerBlock), smem, static_cast<cudaStream_t>(stream), ps,
                         partial, x, w, D, eps, h, state, dev_err);
}

int32_t mb_peer_argmax(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                       const uint16_t* logits, int32_t N, int32_t V, int32_t col0, int32_t* ids, uint32_t* state,
                       uint32_t* dev_err, void* stream) {
  if (!bufs || !logits || !ids || !state) return MB_ERR_NULL;
  if (N < 1 || N > kPeerMaxRows || V < 1 || col0 < 0 || static_cast<int64_t>(col0) + V > 0x7FFFFFFFll)
    return MB_ERR_ARGS;
  PeerSet ps;
  if (!make_peer_set(bufs, world, rank, slot_elems, timeout_ns, &ps)) return MB_ERR_ARGS;
  return launch_with_pdl(k_peer_argmax, dim3(N), dim3(kPeerArgBlock), 0, static_cast<cudaStream_t>(stream), ps, logits,
                         V, col0, ids, state, dev_err);
}

}  // extern "C"
