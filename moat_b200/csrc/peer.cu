// Tensor-parallel exchanges of the decode step over NVLink peer memory (B200, sm_100a).
//
// A row-parallel projection (o_proj, down) leaves on every rank a partial product
// [N, D]; the next operation is the residual add and RMSNorm of the sum over ranks
// (transformer.py:148-158 on one device). A column-split lm_head leaves per rank the
// logits of its vocabulary range; the greedy choice is the argmax over all of them
// (batch_generator.py:203-206, 224-227). Instead of a library all-reduce followed by
// separate kernels, each exchange here is ONE kernel per rank that stores its rows
// straight into the other ranks' exchange buffers (plain peer stores over NVLink, no
// multicast), waits (bounded) for every rank's rows and finishes the operation
// locally:
//   k_peer_add_rmsnorm : sum the N x D partials in rank order in fp32, round to fp16
//                        (the all-reduced projection), x += it, h = RMSNorm(x) * w;
//   k_peer_argmax      : best (value, column) key of this rank's logits row, exchanged,
//                        integer max over ranks -> token id.
// When the projection is the fused GEMM of mb_int4_gemm_peer (gemm.cu), its epilogue
// has already stored this rank's rows as exchange words, and the join
// (k_peer_add_rmsnorm<true>, mb_peer_sum_rmsnorm) only waits, sums and normalises.
// Every rank sums the same values in the same order, so the residual streams stay
// bit-identical across ranks.
//
// Exchange buffer (one per rank, cudaMalloc + CUDA IPC, zeroed at creation), written
// by the other ranks with 8-byte "low-latency" words: 4 bytes of payload and 4 bytes
// holding the epoch of the call that wrote them, stored in one transaction, so a
// receiver that reads a word carrying the current epoch has its payload too (no fence,
// no separate flag, one NVLink crossing per word). Layout in peer_ll.cuh: channel 1
// holds the argmax keys, channel 0 the rows of the residual joins.
// Epoch e (1, 2, ...) of a channel writes parity e & 1; a rank can only reach epoch
// e + 2 after every rank has finished epoch e + 1, hence finished reading epoch e's
// parity, so two parities never race. Each row's epoch lives in a small local state
// array (one word per row and channel, not shared) and is stored by that row's CTA at
// the end of each call, which keeps a captured CUDA graph replayable.
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
#include "peer_ll.cuh"

namespace mb {

constexpr int kPeerBlock = 256;

struct PeerSet {
  uint8_t* buf[kPeerMaxRanks];  // every rank's exchange buffer as mapped in this process (own included)
  int world;
  int rank;
  int64_t slot_elems;  // fp16 elements of one channel-0 slot (>= N * D)
  int64_t timeout_ns;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// The payload of word `p` once it carries `epoch`; waits at most until `deadline`
// (global ns), then sets MB_DEVERR_TIMEOUT and returns whatever the word holds.
__device__ __forceinline__ uint32_t wait_ll(const uint2* p, uint32_t epoch, uint64_t& deadline, int64_t timeout_ns,
                                            uint32_t* err) {
  uint2 v = ld_ll(p);
  if (v.y == epoch) return v.x;
  if (deadline == 0) deadline = global_ns() + static_cast<uint64_t>(timeout_ns);
  while (v.y != epoch) {
    if (global_ns() > deadline) {
      if (err) atomicOr(err, MB_DEVERR_TIMEOUT);
      deadline = 1;  // expired: later words of this call do not wait again
      break;
    }
    v = ld_ll(p);
  }
  return v.x;
}

// Every row keeps its own epoch word: both ranks make the same calls, so CTA n sees
// the same epoch sequence everywhere, and the next call's CTA n reads the word only
// after griddepcontrol.wait (this grid has completed and its writes are visible):
// no fence, no arrival count.
__device__ __forceinline__ void peer_finish(uint32_t* state, uint32_t epoch) {
  if (threadIdx.x == 0) state[blockIdx.x] = epoch;
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

// One CTA per row n. state = the rows' epochs of channel 0. STORED: every rank's rows
// of this epoch were stored by its GEMM's epilogue (partial unused).
template <bool STORED>
__global__ void __launch_bounds__(kPeerBlock) k_peer_add_rmsnorm(PeerSet ps, const uint16_t* __restrict__ partial,
                                                                 float* __restrict__ x, const float* __restrict__ w,
                                                                 int D, float eps, uint16_t* __restrict__ h,
                                                                 uint32_t* state, uint32_t* err) {
  extern __shared__ float delta[];  // [D]: the all-reduced row, fp16-rounded, as float
  __shared__ float part[kPeerBlock / 32];
  pdl_wait();               // the partial and the epoch state come from earlier kernels
  pdl_launch_dependents();  // the next kernel's prologue may overlap; it waits for this grid before reading x, h
  const int n = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(state + n) + 1u;
  const int par = epoch & 1u;
  const int chunks = D / 8;  // 16-byte chunks of a row: four words each
  // this thread's residual and norm-weight values, loaded before the exchange so that
  // their latency hides behind it (the element order of the sum below is unchanged)
  constexpr int kPre = 16;  // D <= 4096 in registers; larger rows read the rest later
  float* xr = x + static_cast<int64_t>(n) * D;
  float xv[kPre], wv[kPre];
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int c = threadIdx.x + j * kPeerBlock;
    xv[j] = c < D ? xr[c] : 0.0f;
    wv[j] = c < D ? w[c] : 0.0f;
  }
  auto slot = [&](uint8_t* buf, int src) {
    return peer_row_slot(buf, par, src, ps.slot_elems) + static_cast<int64_t>(n) * D / 2;
  };
  // 1. this rank's row n as low-latency words into slot [par][rank] of every rank
  if constexpr (!STORED) {
    const uint4* src = reinterpret_cast<const uint4*>(partial + static_cast<int64_t>(n) * D);
    for (int i = threadIdx.x; i < chunks; i += kPeerBlock) {
      const uint4 v = src[i];
      for (int q = 0; q < ps.world; ++q) {
        uint2* d = slot(ps.buf[q], ps.rank) + 4 * i;
        st_ll(d, v.x, epoch);
        st_ll(d + 1, v.y, epoch);
        st_ll(d + 2, v.z, epoch);
        st_ll(d + 3, v.w, epoch);
      }
    }
  }
  // 2. every rank's words of the same chunks (own buffer), summed in rank order in fp32,
  //    one fp16 rounding
  uint64_t deadline = 0;
  for (int i = threadIdx.x; i < chunks; i += kPeerBlock) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    for (int q = 0; q < ps.world; ++q) {
      const uint2* s0 = slot(ps.buf[ps.rank], q) + 4 * i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t word = wait_ll(s0 + j, epoch, deadline, ps.timeout_ns, err);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&word));
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) delta[8 * i + j] = __half2float(__float2half_rn(acc[j]));
  }
  __syncthreads();
  // 3. residual add and RMSNorm, element order as k_add_rmsnorm
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int c = threadIdx.x + j * kPeerBlock;
    if (c < D) {
      const float v = xv[j] + delta[c];
      xv[j] = v;
      xr[c] = v;
      ss = fmaf(v, v, ss);
    }
  }
  for (int c = threadIdx.x + kPre * kPeerBlock; c < D; c += kPeerBlock) {
    const float v = xr[c] + delta[c];
    xr[c] = v;
    ss = fmaf(v, v, ss);
  }
  const float inv = rsqrtf(block_sum_fixed(ss, part) / static_cast<float>(D) + eps);
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int c = threadIdx.x + j * kPeerBlock;
    if (c < D) h[static_cast<int64_t>(n) * D + c] = __half_as_ushort(__float2half_rn(xv[j] * inv * wv[j]));
  }
  for (int c = threadIdx.x + kPre * kPeerBlock; c < D; c += kPeerBlock)
    h[static_cast<int64_t>(n) * D + c] = __half_as_ushort(__float2half_rn(xr[c] * inv * w[c]));
  peer_finish(state, epoch);
}

// One CTA per row n: key of this rank's best logit, exchanged, max over ranks -> ids[n].
// state = the rows' epochs of channel 1.
constexpr int kPeerArgBlock = 1024;

__global__ void __launch_bounds__(kPeerArgBlock) k_peer_argmax(PeerSet ps, const uint16_t* __restrict__ logits, int V,
                                                               int col0, int32_t* __restrict__ ids, uint32_t* state,
                                                               uint32_t* err) {
  __shared__ unsigned long long best_w[kPeerArgBlock / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(state + n) + 1u;
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
    return reinterpret_cast<uint2*>(buf + kPeerKeyOff) + 2 * ((par * kPeerMaxRanks + src) * kPeerMaxRows + n);
  };
  __shared__ unsigned long long got[kPeerMaxRanks];
  if (threadIdx.x < ps.world) {
    unsigned long long b = best_w[0];
    for (int i = 1; i < kPeerArgBlock / 32; ++i) b = best_w[i] > b ? best_w[i] : b;
    uint2* d = key_slot(ps.buf[threadIdx.x], ps.rank);
    st_ll(d, static_cast<uint32_t>(b), epoch);
    st_ll(d + 1, static_cast<uint32_t>(b >> 32), epoch);
    // rank threadIdx.x's key for this row, from this rank's buffer
    uint64_t deadline = 0;
    const uint2* s0 = key_slot(ps.buf[ps.rank], threadIdx.x);
    const uint32_t lo = wait_ll(s0, epoch, deadline, ps.timeout_ns, err);
    const uint32_t hi = wait_ll(s0 + 1, epoch, deadline, ps.timeout_ns, err);
    got[threadIdx.x] = (static_cast<unsigned long long>(hi) << 32) | lo;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int q = 0; q < ps.world; ++q) b = got[q] > b ? got[q] : b;
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
  const size_t slot = static_cast<size_t>(max_rows) * D;  // fp16 elements; two per 8-byte word
  return kPeerRowOff + 2 * kPeerMaxRanks * (slot / 2) * sizeof(uint2);
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

static int32_t peer_join(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                         const uint16_t* partial, float* x, const float* w, int32_t N, int32_t D, float eps,
                         uint16_t* h, uint32_t* state, uint32_t* dev_err, void* stream) {
  if (N < 1 || N > kPeerMaxRows || D < 8 || D % 8 != 0 || static_cast<int64_t>(N) * D > slot_elems ||
      D > 16384)
    return MB_ERR_ARGS;
  if (partial && !aligned(partial, 16)) return MB_ERR_ALIGN;
  PeerSet ps;
  if (!make_peer_set(bufs, world, rank, slot_elems, timeout_ns, &ps)) return MB_ERR_ARGS;
  const size_t smem = static_cast<size_t>(D) * sizeof(float);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (partial) {
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k_peer_add_rmsnorm<false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem)) != cudaSuccess)
      return MB_ERR_LAUNCH;
    return launch_with_pdl(k_peer_add_rmsnorm<false>, dim3(N), dim3(kPeerBlock), smem, st, ps, partial, x, w, D,
                           eps, h, state, dev_err);
  }
  if (smem > 48 * 1024 && cudaFuncSetAttribute(k_peer_add_rmsnorm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem)) != cudaSuccess)
    return MB_ERR_LAUNCH;
  return launch_with_pdl(k_peer_add_rmsnorm<true>, dim3(N), dim3(kPeerBlock), smem, st, ps, partial, x, w, D, eps, h,
                         state, dev_err);
}

int32_t mb_peer_add_rmsnorm(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                            const uint16_t* partial, float* x, const float* w, int32_t N, int32_t D, float eps,
                            uint16_t* h, uint32_t* state, uint32_t* dev_err, void* stream) {
  if (!bufs || !partial || !x || !w || !h || !state) return MB_ERR_NULL;
  return peer_join(bufs, world, rank, slot_elems, timeout_ns, partial, x, w, N, D, eps, h, state, dev_err, stream);
}

int32_t mb_peer_sum_rmsnorm(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                            float* x, const float* w, int32_t N, int32_t D, float eps, uint16_t* h, uint32_t* state,
                            uint32_t* dev_err, void* stream) {
  if (!bufs || !x || !w || !h || !state) return MB_ERR_NULL;
  return peer_join(bufs, world, rank, slot_elems, timeout_ns, nullptr, x, w, N, D, eps, h, state, dev_err, stream);
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
