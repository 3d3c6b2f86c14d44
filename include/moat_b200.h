/*
 * moat_b200 — C ABI of the B200 (sm_100a) INT4 super-block GEMM and exp-LUT
 * decode-attention path.
 *
 * Conventions (after the reference C ABI, antigravity-engine/src/antigravity_c_api.h):
 *   - every entry point returns an int32 status: 0 = ok, < 0 = error detected on the
 *     host before anything was launched (the reference uses -1 for a null / unloaded
 *     context and -2 for invalid arguments, antigravity_c_api.h:129-130);
 *   - the caller owns every buffer (antigravity_c_api.h:76-83, 131-143); all pointers
 *     are DEVICE pointers except the host buffers of mb_int4_gemm_host and
 *     mb_int4_gemm_host_overlap; nothing here allocates device memory (the overlapped
 *     host calls create two copy streams and a few events per caller stream, once);
 *   - work is enqueued asynchronously on the caller's stream (`stream` is a
 *     cudaStream_t; NULL = legacy default stream). The reference is synchronous
 *     (waitUntilCompleted); callers that need the result on the host synchronise;
 *   - fp16 data travels as uint16_t bit patterns; the packed weight format is the
 *     reference's 144-byte super-block (struct SuperBlock, batched_gemm.metal:17-20):
 *     bytes 0..15 = 8 little-endian fp16 group scales, bytes 16..143 = 128 nibble
 *     bytes, byte j = element 2j (low nibble) | element 2j+1 (high nibble), each q+8.
 *     Super-block i holds flat elements [256 i, 256 i + 256) of the row-major [K, M]
 *     weight, W[k, m] at flat index k*M + m.
 *   - stateless and thread-safe; a kernel that needs scratch (decode attention)
 *     takes a caller-owned workspace whose size is given by the matching
 *     *_workspace_size() query; it needs no initial contents, but one workspace
 *     must not be used by two calls that may run concurrently.
 */
#ifndef MOAT_B200_H
#define MOAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MB_OK 0
#define MB_ERR_NULL (-1)        /* a required pointer is NULL */
#define MB_ERR_ARGS (-2)        /* invalid sizes / shapes */
#define MB_ERR_WORKSPACE (-3)   /* workspace too small */
#define MB_ERR_LAUNCH (-4)      /* the CUDA launch itself failed */
#define MB_ERR_ALIGN (-5)       /* a pointer is not 16-byte aligned */
#define MB_ERR_UNSUPPORTED (-6) /* shape outside what this build supports */

/* Device-side error word bits (written to a caller-provided device word). */
#define MB_DEVERR_TIMEOUT 1u /* a bounded wait gave up */
#define MB_DEVERR_INDEX 2u   /* a device-side index (token id, position) was out of range */
#define MB_DEVERR_NONFINITE 4u /* a sampled row had a non-finite (scaled) maximum logit */

#define MB_ABI_VERSION 1

/* ABI version of this library (no reference counterpart; for the ctypes binding). */
int32_t mb_abi_version(void);

/* Human-readable text for a status code. */
const char* mb_status_string(int32_t status);

/* ---------------------------------------------------------------------------
 * INT4 group-32 quantization and super-block packing.
 * Replaces quantize_weights_int4 (antigravity-engine/src/dequant.py:22-60) when
 * variant == 0 ("engine": the fp32 scale max|w|/7 is rounded to fp16 first and
 * the weights are divided by that fp16 scale), and quantize_fp16_to_int4
 * (src/dequant.py:26-55) when variant == 1 ("top-level": divide by the unrounded
 * fp32 scale, then store it as fp16). Round half to even, clip to [-8, 7]; a zero
 * group gets scale 1.0. Also replaces repack_to_superblocks
 * (antigravity-engine/src/dequant.py:69-132) by writing the 144-byte stream.
 *   w        n weights, fp32 (w_is_fp16 = 0) or fp16 bit patterns (w_is_fp16 = 1)
 *   n        multiple of 32; a multiple of 256 if sb_out is given
 *   q_out    optional int8[n]; scales_out optional fp16[n/32]; sb_out optional
 *            uint8[n/256*144]. At least one output must be given.
 * ------------------------------------------------------------------------- */
int32_t mb_int4_quantize(const void* w, int32_t w_is_fp16, int64_t n, int32_t variant, int8_t* q_out,
                         uint16_t* scales_out, uint8_t* sb_out, void* stream);

/* Packs int8 q[n] (values in [-8, 7]) and fp16 scales[n/32] into the 144-byte
 * stream; replaces repack_to_superblocks (antigravity-engine/src/dequant.py:69-132).
 * n must be a multiple of 256. */
int32_t mb_int4_pack(const int8_t* q, const uint16_t* scales, int64_t n, uint8_t* sb_out, void* stream);

/* Super-block stream -> int8 q[nsb*256] and fp16 scales[nsb*8]; replaces
 * unpack_superblock (antigravity-engine/src/dequant.py:135-156). Either output may be NULL. */
int32_t mb_int4_unpack(const uint8_t* sb, int64_t nsb, int8_t* q_out, uint16_t* scales_out, void* stream);

/* ---------------------------------------------------------------------------
 * Dequantization, bit-exact with the reference: out = fp16(q * s), one rounding.
 * mb_int4_dequant replaces unpack_superblock_weights (src/dequant.py:116-147) and
 * the Metal dequantize_superblocks_kernel (batched_gemm.metal:41-66): nsb
 * super-blocks -> fp16[nsb*256].
 * mb_int4_dequant_q replaces lut_dequantize / arithmetic_dequantize
 * (antigravity-engine/src/dequant.py:183-252): int8 q[n] with fp16 scales[n/group]
 * -> fp16[n]; group >= 1, n % group == 0.
 * ------------------------------------------------------------------------- */
int32_t mb_int4_dequant(const uint8_t* sb, uint16_t* out, int64_t nsb, void* stream);
int32_t mb_int4_dequant_q(const int8_t* q, const uint16_t* scales, int64_t n, int32_t group, uint16_t* out,
                          void* stream);

/* Table gather of lut_dequantize_fp16 (src/dequant.py:79-113): out[i] =
 * lut[(i / group_len) % lut_rows][clip(idx[i], 0, lut_cols - 1)], fp16.
 * idx is int32 (already offset the way the reference offsets it). */
int32_t mb_lut_gather_f16(const int32_t* idx, int64_t n, const uint16_t* lut, int64_t lut_rows, int32_t lut_cols,
                          int64_t group_len, uint16_t* out, void* stream);

/* ---------------------------------------------------------------------------
 * Fused INT4 super-block batched GEMM: out[N, M] (fp16) = act[N, K] (fp16, row
 * major) x dequant(sb)[K, M], fp32 accumulation. Replaces the reference's
 * batched_gemm entry point — Metal batched_gemm_simdgroup (batched_gemm.metal:74-109,
 * buffers act/weights/out/N/K/M) and fused_batched_gemm_int4 (:116-169), whose CPU
 * form is the decode step's `activations @ W` (batch_generator.py:290).
 * Requires K*M % 256 == 0 and N >= 1; any N (rows are processed in blocks of 32
 * per launch, or of 16 where only 16 rows fit the fast plan's shared memory). No
 * scratch memory: split-K partial sums are reduced on chip.
 * dev_err is an optional DEVICE word (may be NULL) that receives MB_DEVERR_* bits
 * if a bounded wait inside the kernel gives up. The fast path needs K % 8 == 0,
 * M % 128 == 0 and 16-byte aligned act / sb; other shapes take a slower path.
 * ------------------------------------------------------------------------- */
int32_t mb_int4_gemm(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                     uint32_t* dev_err, void* stream);

/* mb_int4_gemm with HOST activations and output: copies act_host (N x K fp16) into
 * the caller's device staging buffer act_dev, runs the GEMM into out_dev (N x M) and
 * copies it back to out_host, all enqueued on `stream` (cudaMemcpyAsync; pinned host
 * memory makes the copies asynchronous, the caller synchronises before reading
 * out_host). Mirrors the reference C entry point's flow, which writes the host
 * activations into a shared buffer, dispatches the GEMM and waits
 * (antigravity_c_api.cpp:185-220). sb is a DEVICE pointer (weights stay resident);
 * nothing is allocated. */
int32_t mb_int4_gemm_host(const uint16_t* act_host, const uint8_t* sb, uint16_t* out_host, int32_t N, int32_t K,
                          int32_t M, uint16_t* act_dev, uint16_t* out_dev, uint32_t* dev_err, void* stream);

/* Host-buffer GEMM for a stream of calls (the same flow as mb_int4_gemm_host, without
 * its serialisation): the input copy and the output copy of each call run on two
 * library-owned copy streams, ordered with events against `stream` (which runs the
 * GEMM), and each call uses the next of MB_HOST_SLOTS staging slots of `staging`
 * (256-byte aligned, staging_bytes / MB_HOST_SLOTS bytes per slot, at least
 * mb_int4_gemm_host_staging_bytes(N, K, M) / MB_HOST_SLOTS), so consecutive calls'
 * copies overlap their neighbours' GEMMs. Returns once enqueued: out_host is complete,
 * and act_host may be reused, after mb_int4_gemm_host_wait(stream) (or a device
 * synchronise). A slot is rewritten only after its previous output copy finished. */
#define MB_HOST_SLOTS 4
size_t mb_int4_gemm_host_staging_bytes(int32_t N, int32_t K, int32_t M);
int32_t mb_int4_gemm_host_overlap(const uint16_t* act_host, const uint8_t* sb, uint16_t* out_host, int32_t N,
                                  int32_t K, int32_t M, void* staging, size_t staging_bytes, uint32_t* dev_err,
                                  void* stream);
/* Wait on the host for every mb_int4_gemm_host_overlap call enqueued for `stream`. */
int32_t mb_int4_gemm_host_wait(void* stream);

/* Launch plan of the first 32-row block for a shape (introspection, no reference
 * counterpart). info must hold 8 int32: [0] fast path (1) or generic (0), [1] strip
 * width, [2] CTAs per cluster (K split), [3] grid size, [4] pipeline stages, [5]
 * dynamic shared memory bytes, [6] row phases, [7] 8-row batch tiles. */
int32_t mb_int4_gemm_plan(int32_t N, int32_t K, int32_t M, int32_t* info);

/* Columns [c0, c1) of a packed [K, M] weight, re-packed as its own [K, c1-c0]
 * super-block stream (bit-identical q and scales). Column sharding of M across
 * GPUs has no reference counterpart (the reference is single-device); the weight
 * semantics are those of repack_to_superblocks. Needs M % 32 == 0, c0 and c1
 * multiples of 32, K*(c1-c0) % 256 == 0. */
int32_t mb_int4_extract_columns(const uint8_t* sb, int32_t K, int32_t M, int32_t c0, int32_t c1, uint8_t* out,
                                void* stream);

/* ---------------------------------------------------------------------------
 * Exp-LUT softmax and decode attention.
 * `table` is the reference's fp16 exp table (ExponentialLUT.lut,
 * antigravity-engine/src/attention.py:50-51) of `size` entries over [-range_max, 0].
 * mb_exp_lut_lookup replaces ExponentialLUT.lookup (attention.py:60-85):
 *   out[i] = table[size-1-trunc(min(|x| / fp32(range_max/(size-1)), size-1))],
 *   IEEE fp32 divide.
 * mb_lut_softmax replaces safe_softmax_lut (attention.py:97-134) over the last axis
 * of x[rows, cols] (fp32): max-subtract, LUT exp, fp32 sum (zero-sum guard), fp16 out.
 * ------------------------------------------------------------------------- */
int32_t mb_exp_lut_lookup(const uint16_t* table, int32_t size, float range_max, const float* x, int64_t n,
                          uint16_t* out, void* stream);
int32_t mb_lut_softmax(const float* x, int64_t rows, int64_t cols, const uint16_t* table, int32_t size,
                       float range_max, uint16_t* out, void* stream);

/* Decode attention for one query token per (trace, head), LUT softmax:
 *   s_l = (q . k_l) * scale (fp32); p = safe_softmax_lut(s) (fp16); out = sum_l p_l v_l.
 * Composition of gqa_attention_scores_kernel (transformer_ops.metal:94-123),
 * safe_softmax_lut (attention.py:97-134) and attention_value_kernel
 * (transformer_ops.metal:186-214). q [T, H, d], k/v [T, H, L, d], out [T, H, d],
 * all fp16; d a power of two in [8, 256]. The workspace needs no initialisation
 * (the kernels overwrite every byte they read). */
size_t mb_decode_attn_workspace_size(int32_t T, int32_t H, int32_t L, int32_t d);
int32_t mb_decode_attn(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int32_t T,
                       int32_t H, int32_t L, int32_t d, float scale, const uint16_t* table, int32_t size,
                       float range_max, void* workspace, size_t workspace_bytes, void* stream);

/* Decode attention exactly as mb_decode_attn, on a fixed per-device scratch of
 * MB_ATTN_NOALLOC_SCRATCH_BYTES that belongs to the library: the call allocates and
 * frees no device memory. No counterpart in the reference (its attention runs on the
 * host); it serves callers that cannot provide a workspace, such as a binding with no
 * device allocator or a process whose caching allocator already holds the free HBM.
 *   - returns MB_ERR_WORKSPACE, launching nothing, when
 *     mb_decode_attn_workspace_size(T, H, L, d) > MB_ATTN_NOALLOC_SCRATCH_BYTES;
 *   - the scratch needs no zeroing: the kernels write every scratch byte they read;
 *   - all calls on one device share the scratch: calls that may overlap (unordered
 *     streams, several host threads) race and can return wrong outputs;
 *   - the first call on each device looks up the scratch address with that device
 *     current; make it before any stream capture begins on that device. */
#define MB_ATTN_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int32_t mb_decode_attn_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int32_t T,
                               int32_t H, int32_t L, int32_t d, float scale, const uint16_t* table, int32_t size,
                               float range_max, void* stream);

/* Decode attention over a KV cache with room for Lmax positions per (trace, head):
 * k_cache / v_cache [T, H, Lmax, d], the first L positions valid; otherwise exactly
 * mb_decode_attn (same workspace size for (T, H, L, d)). The decode step's attention
 * over its growing cache (reference: Attention.forward with kv_cache,
 * transformer.py:80-121, LUT softmax as in batch_generator.py:226,234). */
int32_t mb_decode_attn_cache(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
                             int32_t T, int32_t H, int32_t L, int32_t Lmax, int32_t d, float scale,
                             const uint16_t* table, int32_t size, float range_max, void* workspace,
                             size_t workspace_bytes, void* stream);

/* mb_decode_attn_cache with the valid length read on the device: trace t uses the
 * first min(Lmax, lens[t] + len_add) positions (lens is a DEVICE int32[T], e.g. the
 * decode positions with len_add = 1), so one captured decode step replays while the
 * cache grows. The grid and the workspace are sized for Lmax
 * (mb_decode_attn_workspace_size(T, H, Lmax, d)). No reference counterpart (the
 * reference passes the length on the host). */
int32_t mb_decode_attn_cache_lens(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
                                  int32_t T, int32_t H, int32_t Lmax, int32_t d, const int32_t* lens, int32_t len_add,
                                  float scale, const uint16_t* table, int32_t size, float range_max, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Decoder-step glue (the element-wise and row-wise operations between the INT4
 * GEMMs of one decode step; reference: antigravity-engine/src/transformer.py).
 * The residual stream x is fp32 [N, D]; GEMM inputs and outputs are fp16.
 * ------------------------------------------------------------------------- */
/* x[n] = fp32(table[ids[n]]) for fp16 table [V, D] (TinyLlamaModel embed_tokens,
 * transformer.py:184, 207). An id outside [0, V) gives a zero row and sets
 * MB_DEVERR_INDEX in the optional device word dev_err. */
int32_t mb_embed(const int32_t* ids, int32_t N, const uint16_t* table, int32_t V, int32_t D, float* x,
                 uint32_t* dev_err, void* stream);

/* x += y (y may be NULL), then h = fp16(x * rsqrt(mean(x^2) + eps) * w): the residual
 * add fused with RMSNorm (transformer.py:26-37, 148-158); w fp32 [D]. */
int32_t mb_add_rmsnorm(float* x, const uint16_t* y, const float* w, int32_t N, int32_t D, float eps, uint16_t* h,
                       void* stream);

/* RoPE on the q and k parts of qkv [N, 3*H*dh] (q | k | v, heads contiguous) at the
 * per-trace positions pos[N] (device), adjacent pairs rotated as in
 * apply_rotary_emb (transformer.py:39-63); cs = fp32 (cos, sin) pairs [Lmax][dh/2].
 * Writes q_out [N, H, dh] and appends k and v at pos into k_cache / v_cache
 * [N, H, Lmax, dh]. A position outside [0, Lmax) skips the row and sets
 * MB_DEVERR_INDEX. */
int32_t mb_rope_append(const uint16_t* qkv, int32_t N, int32_t H, int32_t dh, const int32_t* pos, const float* cs,
                       int32_t Lmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, uint32_t* dev_err,
                       void* stream);

/* a[n, j] = fp16(silu(gu[n, j]) * gu[n, F + j]) for gu [N, 2F] (gate | up), the SwiGLU
 * of SwiGLUMLP.forward (transformer.py:124-134). */
int32_t mb_swiglu(const uint16_t* gu, int32_t N, int32_t F, uint16_t* a, void* stream);

/* ids[n] = first index of the largest value of logits[n, :] (fp16 [N, V]); a NaN
 * counts as the largest, like numpy.argmax (greedy sampling, batch_generator.py:203-206,
 * 224-227). */
int32_t mb_argmax_f16(const uint16_t* logits, int32_t N, int32_t V, int32_t* ids, void* stream);

/* Tensor-parallel greedy choice over a column-split vocabulary (the lm_head shards
 * of a Megatron split; the reference decodes on one device, batch_generator.py:203-206).
 * keys[n] = (c << 32) | (0xFFFFFFFF - (col0 + j)) for the largest logits[n, j] of this
 * shard, c an order-preserving 16-bit code of the fp16 value (NaN largest, -0 == +0),
 * so the int64 MAX over all shards (one all-reduce) is the global argmax with ties to
 * the first column, exactly as mb_argmax_f16 over the whole row. */
int32_t mb_argmax_key_f16(const uint16_t* logits, int32_t N, int32_t V, int32_t col0, int64_t* keys, void* stream);

/* ids[n] = the column encoded in the combined keys[n] of mb_argmax_key_f16. */
int32_t mb_argmax_keys_to_ids(const int64_t* keys, int32_t N, int32_t* ids, void* stream);

/* ---- Tensor-parallel exchanges over NVLink peer memory -------------------------
 * The reference runs on one device; these entry points join the Megatron shards of
 * its decode step (transformer.py:148-158 residual + RMSNorm after o_proj and down;
 * batch_generator.py:203-206 greedy choice after lm_head) without a library
 * collective: each rank stores its rows into every rank's exchange buffer (CUDA IPC
 * mappings, plain peer stores, no multicast) as 8-byte words that each carry 4 bytes
 * of payload and the call's epoch, so a word whose epoch matches is itself the proof
 * that its payload arrived (no fence, no separate flag), and polls its own buffer,
 * bounded by timeout_ns, until every word it reads carries the epoch. Two slot sets
 * alternate by epoch parity, so a fast rank's next call never overwrites words a slow
 * rank has still to read. A wait that expires sets
 * MB_DEVERR_TIMEOUT in dev_err; the outputs of that call are then undefined.
 * bufs[q] is rank q's exchange buffer as mapped in this process (bufs[rank] its own),
 * each of mb_peer_buffer_bytes(max_rows, D) bytes, zeroed before the first call.
 * state is a per-rank DEVICE array of MB_PEER_STATE_WORDS uint32 per exchange kind
 * (zeroed once; every row's epoch lives there, so a captured graph replays). Every
 * rank must make the same sequence of calls, each rank on its own GPU. */
#define MB_PEER_STATE_WORDS 64
#define MB_IPC_HANDLE_BYTES 64

/* Bytes of one exchange buffer for up to max_rows (<= 64) rows of D (multiple of 8)
 * fp16 values and up to 8 ranks; 0 for unsupported sizes. */
size_t mb_peer_buffer_bytes(int32_t max_rows, int32_t D);

/* cudaMalloc(bytes), zero it and write its CUDA IPC handle (MB_IPC_HANDLE_BYTES). */
int32_t mb_ipc_alloc(size_t bytes, void** ptr, uint8_t* handle);
/* Map another process's buffer from its IPC handle (peer access enabled). */
int32_t mb_ipc_open(const uint8_t* handle, void** ptr);
int32_t mb_ipc_close(void* ptr);
int32_t mb_ipc_free(void* ptr);

/* Row-parallel join fused with the next residual add and RMSNorm: with P_q the
 * partial [N, D] fp16 of rank q, y = fp16(sum over q = 0..world-1 of P_q, in rank order
 * in fp32), x += y (fp32 [N, D]) and h = fp16(x * rsqrt(mean(x^2) + eps) * w) as
 * mb_add_rmsnorm; identical x and h on every rank. slot_elems >= N * D (the max_rows
 * * D the buffers were sized for). */
int32_t mb_peer_add_rmsnorm(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                            const uint16_t* partial, float* x, const float* w, int32_t N, int32_t D, float eps,
                            uint16_t* h, uint32_t* state, uint32_t* dev_err, void* stream);

/* Row-parallel projection fused with its join: the GEMM of mb_int4_gemm (this rank's
 * partial [N, M] of a row-split projection, o_proj or down of the reference's
 * transformer.py:148-158 on one device), whose epilogue stores its fp16 rows straight
 * into every rank's exchange buffer as the words mb_peer_add_rmsnorm would store (the
 * same fp16 rounding as mb_int4_gemm's output), so the partial never goes to HBM and
 * the join that follows, mb_peer_sum_rmsnorm with the same state, only waits for the
 * other ranks' rows, sums and normalises. state is read (this call's epoch is
 * state[n] + 1), not advanced: the join advances it. M is the join's D; N <= 64,
 * N * M <= slot_elems. Shapes off the fast GEMM plan (K % 8 != 0, M % 128 != 0,
 * act or sb not 16-byte aligned) return MB_ERR_UNSUPPORTED before any launch: use
 * mb_int4_gemm + mb_peer_add_rmsnorm for those. */
int32_t mb_int4_gemm_peer(const uint16_t* act, const uint8_t* sb, int32_t N, int32_t K, int32_t M,
                          void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, const uint32_t* state,
                          uint32_t* dev_err, void* stream);

/* The join after mb_int4_gemm_peer: mb_peer_add_rmsnorm whose partial rows every rank
 * has already stored through its mb_int4_gemm_peer call of this epoch. */
int32_t mb_peer_sum_rmsnorm(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                            float* x, const float* w, int32_t N, int32_t D, float eps, uint16_t* h, uint32_t* state,
                            uint32_t* dev_err, void* stream);

/* Greedy choice over a column-split vocabulary: this rank holds logits [N, V] of
 * columns [col0, col0 + V); ids[n] = the global first index of the largest logit over
 * all ranks (NaN largest, -0 == +0), as mb_argmax_f16 over the whole row. */
int32_t mb_peer_argmax(void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, int64_t timeout_ns,
                       const uint16_t* logits, int32_t N, int32_t V, int32_t col0, int32_t* ids, uint32_t* state,
                       uint32_t* dev_err, void* stream);

/* ---- Batched sampling (BatchedRolloutCoordinator.sample_tokens, NumPy branch,
 * batch_generator.py:187-253) ----------------------------------------------------
 * logits [N, V] fp16 (logits_f32 = 0) or fp32 (1), device. temperature <= 0: greedy,
 * tokens[n] = first index of the largest logit, logprobs[n] = fp16(log p) with p the
 * fp16 LUT softmax (safe_softmax_lut, attention.py:97-134) of the raw row.
 * temperature > 0: s = logits / max(T, 1e-5) (fp16 logits: fp16 quotient by fp16(T)),
 * p = fp16 LUT softmax of s; the k = min(top_k, V) largest p, ordered by (p desc,
 * column asc), renormalised; the token is the first candidate whose running fp32 sum
 * exceeds u * total; logprobs[n] = log(max(p_token, 1e-10)) (fp32). u is uniforms[n]
 * (device, [0, 1)) if given, else the top 24 bits of splitmix64(splitmix64(seed ^
 * counter * 0xD1B54A32D192ED03) + n) * 2^-24, counter = rng_state[0]. Every call
 * advances rng_state[0] by one on the device (rng_state: 2 uint32, zeroed once), so a
 * captured graph draws fresh values each replay. The table is the exp LUT
 * (ExponentialLUT, attention.py:21-90; the reference sampler uses range_max 10), at
 * most 32768 entries. top_k in [1, 64] (the reference uses 50). A row whose (scaled)
 * maximum is not finite (the reference raises) sets MB_DEVERR_NONFINITE, returns its
 * argmax and a NaN logprob. The workspace holds N * V uint16 table indices. */
size_t mb_sample_workspace_size(int32_t N, int32_t V);
int32_t mb_sample_tokens(const void* logits, int32_t logits_f32, int32_t N, int32_t V, float temperature,
                         int32_t top_k, const uint16_t* table, int32_t size, float range_max, const float* uniforms,
                         uint64_t seed, uint32_t* rng_state, int32_t* tokens, float* logprobs, void* workspace,
                         size_t workspace_bytes, uint32_t* dev_err, void* stream);

/* pos[n] += 1 on the device (the next decode step's positions; no reference
 * counterpart: keeps a captured step replayable). */
int32_t mb_advance_positions(int32_t* pos, int32_t N, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOAT_B200_H */
