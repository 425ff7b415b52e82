/*
 * b2attn.h - C ABI of libb2attn.so, the B200 (sm_100a) attention path for the
 * alpaccaroo inference engine.
 *
 * Three hot kernels sit behind this boundary:
 *   1. single-token GQA decode over the KV cache with split-KV partitions and
 *      a log-sum-exp combine           (b2a_decode, b2a_lse_combine)
 *   2. causal flash prefill on tcgen05 tensor cores with TMEM accumulators
 *                                      (b2a_prefill)
 *   3. fused RoPE (norm / neox / IMROPE) plus KV-cache append
 *                                      (b2a_rope_append, b2a_imrope_append)
 *
 * Conventions (all entry points):
 *   - Every pointer named *_dev, and every tensor argument, is device memory
 *     on the current CUDA device; `stream` is a cudaStream_t (NULL = legacy
 *     default stream).  Nothing here allocates device memory, synchronises
 *     the stream or reads device memory on the host, so every call can be
 *     captured into a CUDA graph.  Lengths and positions that change from
 *     token to token are read from device buffers for the same reason.
 *   - The KV cache keeps the reference layout: per layer and per sequence a
 *     token-major [n_ctx][n_kv][head_dim] block (alpaccaroo/model.py:867-870),
 *     rows addressed by absolute position.  A batch of sequences is a set of
 *     such blocks `seq_stride` elements apart.
 *   - Return value: B2A_OK (0) or a B2A_ERR_* code; b2a_last_error() holds a
 *     message for the calling thread.  Kernels never trap: a bounded device
 *     wait that expires or a position outside the cache records a code that
 *     b2a_device_error() reads back.
 */
#ifndef B2ATTN_H_
#define B2ATTN_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2A_ABI_VERSION 1

/* element types */
#define B2A_F32 0
#define B2A_F16 1
#define B2A_BF16 2

/* RoPE styles (alpaccaroo/model.py:1162-1209: "norm" adjacent pairs, "neox"
 * split halves) */
#define B2A_ROPE_NORM 0
#define B2A_ROPE_NEOX 1

/* status codes */
#define B2A_OK 0
#define B2A_ERR_ARG 1         /* null pointer, negative or zero size        */
#define B2A_ERR_SHAPE 2       /* inconsistent shapes (heads, group, ...)     */
#define B2A_ERR_DTYPE 3       /* unsupported element type combination       */
#define B2A_ERR_ALIGN 4       /* pointer or stride not 16-byte aligned       */
#define B2A_ERR_UNSUPPORTED 5 /* head_dim or group outside the kernels' set  */
#define B2A_ERR_WORKSPACE 6   /* caller workspace too small                  */
#define B2A_ERR_CUDA 7        /* CUDA runtime / driver error at launch       */
#define B2A_ERR_TIMEOUT 8     /* device: a bounded wait expired              */
#define B2A_ERR_POSITION 9    /* device: position outside cache or table     */

/* ---- library ---------------------------------------------------------- */

int b2a_version(void);
const char* b2a_last_error(void);

/* Read (and with clear != 0, reset) the device error record of the current
 * device.  Synchronises the device.  *code = 0 means no kernel reported. */
int b2a_device_error(int* code, int* aux, int clear);

/* No reference counterpart: a self-test of the bounded device waits.  Launches
 * one thread that waits on an mbarrier nothing arrives on; after the library's
 * wait limit (2 s) the wait records B2A_ERR_TIMEOUT (aux 0x7F000) and the
 * kernel returns, leaving the context usable.  Read the record with
 * b2a_device_error. */
int b2a_selftest_wait_timeout(void* stream);

/* Launch mode of the calling thread's later launches; returns the previous
 * flags.  B2A_LAUNCH_PDL launches b2a_rope_append, b2a_imrope_append,
 * b2a_decode (both kernels), b2a_lse_combine, b2a_gemm and b2a_gemm_qkv_rope as
 * programmatic dependents of the kernel before them on the stream: each
 * starts while that kernel drains and waits for it (griddepcontrol.wait)
 * before reading what it wrote.  The decode's K/V rows below the newest
 * (row len - 1 of each sequence) are streamed before that wait, and every
 * kernel reads lens_dev / positions before it, so those, and the older
 * cache rows, must be complete before the preceding kernel starts (host
 * copies or earlier kernels), as in a decode step whose RoPE + append
 * writes the newest row.  For captured chains of steps; 0 is the default. */
#define B2A_LAUNCH_PDL 1
int b2a_set_launch_flags(int flags);

/* ---- (1) split-KV GQA decode ------------------------------------------
 *
 * Replaces Model._attention_np (alpaccaroo/model.py:1231-1252),
 * kernels.attention_decode (alpaccaroo/kernels.py:1183-1200),
 * qwen35_kernels.qwen35_full_attention_decode (qwen35_kernels.py:363-392) and
 * the device pair _attention_decode_part/_attention_decode_combine
 * (alpaccaroo/cuda.py:580-694, kernel table cuda.py:967-981).
 *
 *   q        f32 [B][H][D]        one query token per sequence
 *   k_cache  kv_dtype, sequence b at k_cache + b*seq_stride, [n_ctx][KV][D]
 *   v_cache  same layout as k_cache
 *   lens_dev int32 [B]            logical length of each sequence (rows
 *                                 0..len-1 are attended; 0 gives out = 0 and
 *                                 lse = -inf)
 *   out      f32 [B][H][D]        softmax(q.K^T * scale) . V
 *   lse_out  f32 [B][H] or NULL   natural-log log-sum-exp of the scaled
 *                                 scores, for b2a_lse_combine across shards
 *   max_len  host upper bound on every lens_dev entry (<= n_ctx); sizes the
 *            fixed launch grid so a captured graph replays for any lengths
 *   split_rows  KV rows per CTA (multiple of 64), 0 = library choice
 * Head h reads KV head h / (H / KV) (contiguous grouping, qwen35_ops.py:406-
 * 472).  kv_dtype F16/BF16 runs the TMA + tensor-core kernel (D in {64, 128,
 * 256}, H/KV <= 16); F32 runs an fp32 FMA kernel (D % 32 == 0, D <= 256). */
size_t b2a_decode_workspace_bytes(int B, int H, int D, int max_len, int split_rows);
int b2a_decode_split_rows(int B, int KV, int max_len, int kv_dtype);
int b2a_decode(const float* q, const void* k_cache, const void* v_cache, const int* lens_dev,
               float* out, float* lse_out, void* workspace, size_t workspace_bytes, int B, int H,
               int KV, int D, int n_ctx, long long seq_stride, int kv_dtype, float scale,
               int max_len, int split_rows, void* stream);

/* Decode without any device allocation. This entry point has no counterpart
 * in the reference.  It is for callers that can't call cudaMalloc: a serving
 * process that reserved nearly all of HBM for its KV cache up front, a host
 * whose allocator owns every device buffer, or an FFI host with no device
 * allocator.  Same arguments and results as b2a_decode, minus the workspace:
 * the split partials live in one static device array of
 * B2A_DECODE_NOALLOC_SCRATCH_BYTES (16 MiB), which every GPU that loads the
 * library holds until the process exits.
 *   - A call whose partials (b2a_decode_workspace_bytes) exceed the array is
 *     rejected with B2A_ERR_WORKSPACE; a larger split_rows needs less.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - All calls share the array and it keeps the last call's contents: calls
 *     that overlap on the GPU (two streams, or two threads without ordering)
 *     race on it.  Nothing in it needs to start at zero. */
#define B2A_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)
int b2a_decode_noalloc(const float* q, const void* k_cache, const void* v_cache,
                       const int* lens_dev, float* out, float* lse_out, int B, int H, int KV,
                       int D, int n_ctx, long long seq_stride, int kv_dtype, float scale,
                       int max_len, int split_rows, void* stream);

/* Merge G partial decodes of the same queries over disjoint KV ranges (the
 * long-context shard combine).  Same algebra as _attention_decode_combine
 * (alpaccaroo/cuda.py:674-694) with normalised parts:
 *   out[r] = sum_g exp(lse[g][r] - L) * o[g][r],  L = log sum_g exp(lse[g][r])
 * Part g's o rows start at o_parts + g*o_part_stride ([rows][D] f32) and its
 * lse at lse_parts + g*lse_part_stride ([rows] f32); a stride of 0 means
 * dense ([G][rows][D], [G][rows]), so one gathered buffer holding each rank's
 * o followed by its lse can be read in place.  lse_out may be NULL. */
int b2a_lse_combine(const float* o_parts, long long o_part_stride, const float* lse_parts,
                    long long lse_part_stride, int G, int rows, int D, float* out,
                    float* lse_out, void* stream);

/* ---- long-context decode sharded across GPUs ---------------------------
 *
 * The KV rows of every sequence are split into contiguous ranges, one per
 * GPU (rank); each rank calls b2a_decode_sharded on its range and every
 * rank receives the merged result.  Replaces, for a context too long for
 * one GPU, b2a_decode followed by an all-gather of the per-rank (o, lse)
 * parts and b2a_lse_combine: the algebra of _attention_decode_combine
 * (alpaccaroo/cuda.py:674-694) lifted from split CTAs to ranks.  The
 * reference has no multi-GPU decode; this is the natural shard of its
 * split-KV decode.
 *
 * One kernel after the split kernel merges this rank's splits per row,
 * stores the row (o, lse) into every rank's exchange buffer over NVLink
 * (plain peer stores through CUDA-IPC mappings, each value in an 8-byte
 * word with the step number as its tag, so no fence or flag is needed),
 * waits until every rank's words of the row carry this step's tag
 * (bounded: on expiry B2A_ERR_TIMEOUT is recorded) and merges the G parts
 * by their lse.
 *
 *   q, k_shard, v_shard, lens_dev, out, lse_out, workspace, sizes, dtype,
 *   scale, max_len, split_rows  as in b2a_decode, over this rank's rows
 *   peer_xbufs_dev  device array [G] of pointers: rank g's exchange buffer
 *                   as mapped in this process (this rank's own at [rank])
 *   rank, G         this rank and the number of ranks (G <= 128)
 * Exchange buffers: b2a_shard_exchange_bytes(B, H, D, G) bytes per rank,
 * zeroed once, then mapped by every rank (b2a_ipc_handle / b2a_ipc_open)
 * before any rank's first call.  Every rank makes the same sequence of
 * calls with the same B, H and D; a rank's call completes only when every
 * rank's call for the same step has published its rows, so the G calls of
 * a step must be able to run at the same time (one process per GPU).  The
 * call can be captured in a CUDA graph (step counters live on the device). */
size_t b2a_shard_exchange_bytes(int B, int H, int D, int G);
int b2a_decode_sharded(const float* q, const void* k_shard, const void* v_shard,
                       const int* lens_dev, float* out, float* lse_out, void* workspace,
                       size_t workspace_bytes, int B, int H, int KV, int D, int n_ctx,
                       long long seq_stride, int kv_dtype, float scale, int max_len,
                       int split_rows, void* const* peer_xbufs_dev, int rank, int G,
                       void* stream);

/* CUDA IPC plumbing for the exchange buffers (set-up only; no reference
 * counterpart).  b2a_ipc_handle writes the B2A_IPC_HANDLE_BYTES-byte handle
 * of the allocation holding dev_ptr and dev_ptr's offset inside it;
 * b2a_ipc_open maps a peer process's handle (peer access enabled lazily)
 * and returns the mapping's base and base + offset; b2a_ipc_close unmaps a
 * base returned by b2a_ipc_open.  The allocation must come from cudaMalloc
 * (PyTorch's default caching allocator qualifies; expandable segments do
 * not). */
#define B2A_IPC_HANDLE_BYTES 64
int b2a_ipc_handle(const void* dev_ptr, void* handle_out, long long* offset_out);
int b2a_ipc_open(const void* handle, long long offset, void** base_out, void** ptr_out);
int b2a_ipc_close(void* base);

/* ---- (2) causal prefill on tcgen05 --------------------------------------
 *
 * Replaces Model._attention_batch_np (alpaccaroo/model.py:1254-1272), its
 * window variant _attention_batch_window_np (model.py:1567-1592),
 * cuda.attention_batch / _attention_batch_gqa (alpaccaroo/cuda.py:424-578,
 * 1186-1242) and qwen35_full_attention_prefill (qwen35_kernels.py:395-411).
 *
 *   q        in_dtype [T][H][D]   rotated queries (F32, F16 or BF16)
 *   k_cache  in_dtype [t_kv][KV][D] rows kv_start .. kv_start+t_kv-1
 *   v_cache  same
 *   pos_dev  int32 [T]            absolute position of each query token
 *   out      out_dtype [T][H][D]  (F32, F16 or BF16)
 * Key s (absolute position kv_start+s) is visible to query t iff
 * kv_start+s <= pos[t] and (window <= 0 or kv_start+s > pos[t]-window).
 * A query row with no visible key gets the mean of the t_kv value rows of
 * its KV head, the NumPy path's result (its -1e30 mask weighs every key
 * equally).
 *   F16 / BF16 inputs: tcgen05 tensor cores, fp32 accumulation, P rounded
 *     to the input type; D in {64, 128, 256}; positions non-decreasing
 *     within each 128-token tile (a row outside its tile's key range
 *     records B2A_ERR_POSITION).
 *   F32 inputs: fp32 products and accumulation on the CUDA cores (the
 *     reference's precision); D a multiple of 4, at most 256; positions in
 *     any order. */
int b2a_prefill(const void* q, const void* k_cache, const void* v_cache, const int* pos_dev,
                void* out, int T, int t_kv, int H, int KV, int D, int in_dtype, int out_dtype,
                float scale, int window, int kv_start, void* stream);

/* ---- (3) fused RoPE + KV append ----------------------------------------
 *
 * Replaces _rope_np / _rope_batch_np plus the cache-row stores
 * (alpaccaroo/model.py:1162-1209, 1331-1337, 1429-1432), kernels.rope_decode
 * (kernels.py:1172-1180) and the device kernels _rope_store_decode /
 * _rope_store_batch (alpaccaroo/cuda.py:723-786, 885-953).
 *
 * For each token i (0..n_tok-1) at position p = pos_dev[i]:
 *   q row  q + i*q_tok_stride      [H][D] f32, plus bq if non-NULL, rotated;
 *          written to q_out (+ i*H*D, q_out_dtype) or, if q_out is NULL, in
 *          place into q
 *   k row  k + i*k_tok_stride      [KV][D] f32 (+bk), rotated, stored at
 *          k_cache row p of sequence s
 *   v row  v + i*v_tok_stride      [KV][D] f32 (+bv), stored at v_cache row p
 * where s = i if tok_seq_mode == 1 (batched decode: one token per sequence)
 * and s = 0 if tok_seq_mode == 0 (a prefill chunk of one sequence).
 * cos_tab / sin_tab are the engine's f32 tables [tab_rows][n_rot/2]
 * (model.py:871-875); products and differences are rounded separately, so
 * f32 results are bit-identical to the NumPy path.  Dims n_rot..D-1 pass
 * through.  A position outside [0, min(n_ctx, tab_rows)) writes nothing and
 * records B2A_ERR_POSITION.  KV = 0 (k, v and caches NULL) rotates q only,
 * the contract of kernels.rope_decode. */
int b2a_rope_append(float* q, long long q_tok_stride, const float* k, long long k_tok_stride,
                    const float* v, long long v_tok_stride, const float* bq, const float* bk,
                    const float* bv, const float* cos_tab, const float* sin_tab, int tab_rows,
                    const int* pos_dev, int tok_seq_mode, void* k_cache, void* v_cache,
                    long long seq_stride, int n_ctx, int kv_dtype, void* q_out, int q_out_dtype,
                    int n_tok, int H, int KV, int D, int n_rot, int style, void* stream);

/* IMROPE variant for the Qwen35 full-attention layers (qwen35_ops.py:138-215,
 * qwen35_cuda.py:965-1008): pair j < sum(sections) rotates dims (j,
 * j+sum(sections)) by theta = lanes[lane(j)] * freq_scale *
 * freq_base^(-2j / (2*sum(sections))), lane(j) the interleaved T/H/W/E
 * schedule, evaluated in double precision like the reference.
 *   lanes_dev int32 [n_tok][4] position lanes ([p,p,p,0] for text)
 *   sections  host int[4]
 * Cache row, q/k/v and output arguments as in b2a_rope_append. */
int b2a_imrope_append(const float* q, long long q_tok_stride, const float* k,
                      long long k_tok_stride, const float* v, long long v_tok_stride,
                      const int* lanes_dev, const int* sections, double freq_base,
                      double freq_scale, const int* pos_dev, int tok_seq_mode, void* k_cache,
                      void* v_cache, long long seq_stride, int n_ctx, int kv_dtype, void* q_out,
                      int q_out_dtype, int n_tok, int H, int KV, int D, void* stream);

/* Convert n cache elements between storage types, on the device: widening
 * a 16-bit cache to f32 (exact) for a snapshot or a host f32 mirror, and
 * narrowing f32 rows to 16 bits (round to nearest even) for a restore or a
 * mirror upload.  Replaces the host-side conversions around the reference's
 * device KV mirror: the f32 -> f16 staging of _sync_mirror
 * (alpaccaroo/cuda.py:1881-1900) and the f16 -> f32 widening of rows coming
 * home after a device prefill chunk (cuda.py:2046-2061).  Snapshots keep
 * the reference's f32-le row format (alpaccaroo/memory.py:224-241).
 *
 *   src, dst  device buffers of n elements (any of F32/F16/BF16 each; same
 *             type is a copy); they must not overlap
 * Returns B2A_OK or B2A_ERR_ARG / B2A_ERR_DTYPE / B2A_ERR_CUDA. */
int b2a_kv_convert(const void* src, int src_dtype, void* dst, int dst_dtype, long long n,
                   void* stream);

/* Qwen35 full-attention prologue for n_tok tokens (the part of
 * Qwen35Model._attention between the projections and the attention read,
 * alpaccaroo/qwen35_runtime.py:606-646; device kernels split_query_gate,
 * rms_norm, imrope, kv_append of qwen35_cuda.py:907-1008, wired in
 * qwen35_cuda_graph.py:781-829).  For each token and head:
 *   q_h = IMROPE(RMSNorm(query part of query_gate row h, q_norm))  -> q_out
 *   k_g = IMROPE(RMSNorm(key row g, k_norm))  -> k_cache row pos (head g)
 *   v_g                                       -> v_cache row pos (head g)
 * RMSNorm is x / sqrt(mean(x^2) + epsilon) * w, evaluated in double relative
 * to max(|x|, sqrt(epsilon)) and rounded to f32 (qwen35_ops.py:46-75);
 * IMROPE is b2a_imrope_append's rotation (pairs (j, j+P), P = sum(sections)).
 *
 *   query_gate f32 [n_tok] rows of [H][ query(D) | gate(D) ], qg_tok_stride apart
 *   key, value f32 [n_tok] rows of [KV][D]
 *   q_norm, k_norm f32 [D]
 *   lanes_dev  int32 [n_tok][4] position lanes ([p,p,p,0] for text)
 *   pos_dev    int32 [n_tok]    cache row of each token
 *   q_out      [n_tok][H][D] of q_out_dtype
 * Caches and tok_seq_mode as in b2a_rope_append.  D even, <= 256; H a
 * multiple of KV.  The gates stay in query_gate for b2a_sigmoid_gate. */
int b2a_qwen35_attn_prep(const float* query_gate, long long qg_tok_stride, const float* key,
                         long long k_tok_stride, const float* value, long long v_tok_stride,
                         const float* q_norm, const float* k_norm, double epsilon,
                         const int* lanes_dev, const int* sections, double freq_base,
                         double freq_scale, const int* pos_dev, int tok_seq_mode, void* k_cache,
                         void* v_cache, long long seq_stride, int n_ctx, int kv_dtype,
                         void* q_out, int q_out_dtype, int n_tok, int H, int KV, int D,
                         void* stream);

/* out[r][c] = values[r][c] * sigmoid(gates[r][c]) for rows x width f32
 * elements, each array with its own row stride (elements); evaluated in
 * double and rounded to f32 (the attention output gate of
 * qwen35_runtime.py:652-659 with tensor.py:123-129's stable sigmoid; device
 * kernel sigmoid_gate, qwen35_cuda.py:953-963).  For a Qwen35 layer the gates
 * are read in place: gates = query_gate + D, gate_row_stride = 2*D. */
int b2a_sigmoid_gate(const float* values, long long value_row_stride, const float* gates,
                     long long gate_row_stride, float* out, long long out_row_stride, int rows,
                     int width, void* stream);

/* b2a_q8_gemv flags */
#define B2A_GEMV_ACCUMULATE 1 /* out[r] += product (the residual stream) */
#define B2A_GEMV_SWIGLU_OUT 2 /* 16-row groups of 8 gate + 8 up rows: out = silu(gate) * up */
#define B2A_GEMV_PDL 4        /* launch as a programmatic dependent of the previous kernel */

/* Q8_0 matrix-vector product for a decode step (batch 1):
 *   out[r] (=|+=) sum_b d[r][b] * sum_{l<32} q[r][32b+l] * xin[32b+l]
 * the reference's Q8_0 matvec (alpaccaroo/qmatrix.py:312-320, device chain
 * kernel cuda.py:241-286), with the step's input transform fused:
 *   mode 0  xin = x                                        (x: cols f32)
 *   mode 1  xin = x * (1/sqrt(x.x/cols + eps)) * aux       (RMSNorm,
 *           tensor.py:349-356; aux = the norm weight)
 *   mode 2  xin = g / (1 + exp(-g)) * u, g = x[0:cols], u = x[cols:2cols]
 *           (SwiGLU, model.py:1466-1467)
 * flags: B2A_GEMV_ACCUMULATE adds into out (the residual stream);
 * B2A_GEMV_SWIGLU_OUT, for a matrix whose rows interleave the FFN's gate and
 * up rows, writes g/(1+exp(-g))*u of each (gate, up) row pair (rows/2 values);
 * B2A_GEMV_PDL launches the kernel as a programmatic dependent of the
 * previous kernel on the stream: it loads its first weight tiles while
 * that kernel finishes and reads x only after it completed.  Weights are the
 * Q8_0 records repacked once: rows padded to a multiple of 16 and cut into
 * 512-byte tiles of 16 rows x one 32-code block, tile (rg, b) at byte
 * (rg * cols/32 + b) * 512 in mma.sync m16n8k16 A-fragment order (lane t's
 * 16 bytes: rows t/4 and t/4 + 8, codes 2(t%4) + {0, 1, 8, 9}, then + 16);
 * scales f16, 16 per tile in the order (row 0, row 8, row 1, row 9, ...).
 * For B2A_GEMV_SWIGLU_OUT each 16-row group holds 8 gate rows then the
 * matching 8 up rows (rows a multiple of 16).  cols a multiple of 32,
 * <= 16384; tiles, x and aux 16-byte aligned, scales 4-byte aligned. */
int b2a_q8_gemv(const void* codes, const void* scales, int rows, int cols, const float* x,
                const float* aux, int mode, float eps, float* out, int flags, void* stream);

/* A decode step's QKV projection with the RMSNorm in front and RoPE + K/V
 * append in the epilogue: the Q8_0 GEMV of b2a_q8_gemv (mode 1, the
 * attention norm weight norm_w) over the (H + 2*KV)*D rows [q; k; v] of
 * a llama layer, then, at the position *pos_dev (the token's cache row):
 *   q rows  rotated (norm style: pairs 2i, 2i+1 of each head, the
 *           reference's f32 products, model.py:1162-1209) into q_out
 *           (f32 [H*D])
 *   k rows  rotated into k_cache row pos ([n_ctx][KV][D] of kv_dtype)
 *   v rows  into v_cache row pos (model.py:1431-1432)
 * cos_tab / sin_tab f32 [tab_rows][D/2] (model.py:318-323).  flags: 0 or
 * B2A_GEMV_PDL.  A position outside the cache or table records
 * B2A_ERR_POSITION.  One launch instead of the GEMV plus b2a_rope_append. */
int b2a_q8_gemv_qkv_rope(const void* codes, const void* scales, int cols, const float* x,
                         const float* norm_w, float eps, float* q_out, const float* cos_tab,
                         const float* sin_tab, int tab_rows, const int* pos_dev, void* k_cache,
                         void* v_cache, int kv_dtype, int n_ctx, int H, int KV, int D, int flags,
                         void* stream);

/* out[i][c] = q[tok_i][c] * d[tok_i][c/32] for the n_tok tokens read from
 * tokens_dev: dequantized Q8_0 embedding rows (qmatrix.py:445-447;
 * T.matrix_row / matrix_rows at model.py:1396, :1308).  A token outside
 * [0, rows) records B2A_ERR_POSITION. */
int b2a_q8_embed(const void* codes, const void* scales, int rows, int cols,
                 const int* tokens_dev, int n_tok, float* out, void* stream);

/* Row-wise glue of a device-resident prefill chunk (Model.forward_batch,
 * model.py:1274-1372; device prefill_chunk, cuda.py:1943-2080):
 *   b2a_rmsnorm_rows  out[t] = x[t] * (1/sqrt(mean(x[t]^2) + eps)) * w
 *                     (tensor.py:355-356), out in out_dtype (the GEMM input)
 *   b2a_swiglu_rows   out[t][i] = g/(1+exp(-g))*u (model.py:1352-1354) with
 *                     (g, u) = (gu[t][2i], gu[t][2i+1]) when interleaved,
 *                     else (gu[t][i], gu[t][F+i])
 * Strides are in elements; x, w, gu f32. */
int b2a_rmsnorm_rows(const float* x, long long x_row_stride, const float* w, float eps, void* out,
                     long long out_row_stride, int out_dtype, int n_rows, int E, void* stream);
int b2a_swiglu_rows(const float* gu, long long gu_row_stride, int interleaved, void* out,
                    long long out_row_stride, int out_dtype, int n_rows, int F, void* stream);

/* ---- prefill-chunk GEMMs on the tcgen05 tensor cores ---------------------
 *
 * The dense projections of a device-resident prefill chunk (the reference's
 * Model.forward_batch, model.py:1274-1372; device prefill_chunk,
 * cuda.py:1943-2080, whose Q8_0 GEMM is cuda.py:287-422), with 16-bit
 * operands (the dequantized weights d * code) and fp32 accumulation:
 *   B2A_GEMM_STORE   out[m][n] = sum_k a[m][k] * w[n][k] (+ c_in[m][n])
 *   B2A_GEMM_SWIGLU  out[m][128g + j] = silu(s[256g + j]) * s[256g + 128 + j]
 *                    for s = a . w^T: w's rows come in 256-row groups of 128
 *                    gate rows then the matching 128 up rows (model.py:
 *                    1352-1354); out has N / 2 columns, N % 256 == 0, no c_in
 *   B2A_GEMM_SWIGLU8 the same with w's rows in 16-row groups of 8 gate rows
 *                    then their 8 up rows (the decode GEMV's layout), N % 16 == 0
 * a [M][lda] and w [N][ldw] of dtype (B2A_F16 / B2A_BF16), K contiguous;
 * c_in f32 [M][ldc] or NULL (may equal out for an in-place residual add);
 * out [M][ldo] of out_dtype.  Pointers 16-byte aligned; lda, ldw multiples of
 * 8 elements; rows of out and c_in start on 16-byte boundaries. */
#define B2A_GEMM_STORE 0
#define B2A_GEMM_SWIGLU 1
int b2a_gemm(const void* a, long long lda, const void* w, long long ldw, int dtype,
             const float* c_in, long long ldc, void* out, long long ldo, int out_dtype, int M,
             int N, int K, int epilogue, void* stream);

/* A prefill chunk's QKV projection with RoPE and the K/V append in the
 * epilogue: the tcgen05 GEMM of b2a_gemm over the (H + 2*KV)*D rows
 * [q; k; v] of w (a [M][lda], w [N][ldw], both of dtype F16 or BF16), then
 * for each token row m at position pos_dev[m] (model.py:1303-1337; device
 * prefill_chunk, cuda.py:1943-2080 with _rope_store_batch, cuda.py:885-953):
 *   q  rotated (norm style: pairs 2i, 2i+1 of each head, the reference's
 *      f32 products) into q_out [M][H*D] of dtype
 *   k  rotated into k_cache row pos ([n_ctx][KV][D] of dtype)
 *   v  into v_cache row pos
 * cos_tab / sin_tab f32 [tab_rows][D/2]; D a multiple of 32.  A position
 * outside the cache or table records B2A_ERR_POSITION and writes nothing
 * for that token.  One launch instead of b2a_gemm plus b2a_rope_append. */
int b2a_gemm_qkv_rope(const void* a, long long lda, const void* w, long long ldw, int dtype,
                      int M, int K, const int* pos_dev, const float* cos_tab, const float* sin_tab,
                      int tab_rows, int H, int KV, int D, void* q_out, void* k_cache,
                      void* v_cache, int n_ctx, void* stream);

/* The same GEMMs straight from Q8_0 weights, the way the reference's chunk
 * GEMM reads them (the codes-decoding GEMM, cuda.py:287-422, with
 * Q8_0 records of quants.py: a f16 scale d per 32 codes): no 16-bit weight
 * copy exists.  The kernel loads the int8 codes with TMA and converter warps
 * write d * code, rounded once to dtype, into the tensor cores' operand
 * tiles in shared memory, so the product equals b2a_gemm's on the
 * dequantized matrix (bit for bit, except the summation order of an
 * in-place residual split over CTAs).
 *   codes int8 [N][ldq] (row n, code k at n*ldq + k), 16-byte aligned,
 *         ldq >= K and a multiple of 16
 *   scales f16 [N][lds]: the scale of codes 32b..32b+31 of row n at
 *         n*lds + b, lds >= K/32
 * K a multiple of 32.  Epilogues as b2a_gemm's, plus
 *   B2A_GEMM_SWIGLU8 out[m][8g + j] = silu(s[16g + j]) * s[16g + 8 + j]
 *                    (j < 8): rows in 16-row groups of 8 gate rows then the
 *                    matching 8 up rows, the layout b2a_q8_gemv's
 *                    B2A_GEMV_SWIGLU_OUT reads; N % 16 == 0, no c_in. */
#define B2A_GEMM_SWIGLU8 2
int b2a_gemm_q8(const void* a, long long lda, const void* codes, long long ldq,
                const void* scales, long long lds, int dtype, const float* c_in, long long ldc,
                void* out, long long ldo, int out_dtype, int M, int N, int K, int epilogue,
                void* stream);

/* b2a_gemm_qkv_rope from Q8_0 weights (codes and scales as b2a_gemm_q8,
 * N = (H + 2*KV)*D rows [q; k; v]). */
int b2a_gemm_qkv_rope_q8(const void* a, long long lda, const void* codes, long long ldq,
                         const void* scales, long long lds, int dtype, int M, int K,
                         const int* pos_dev, const float* cos_tab, const float* sin_tab,
                         int tab_rows, int H, int KV, int D, void* q_out, void* k_cache,
                         void* v_cache, int n_ctx, void* stream);

/* Q8_0 rows to 16-bit rows on the device: out[r][k] = d[r][k/32] * code[r][k]
 * rounded once to dtype (F16 or BF16), the element b2a_gemm_q8 feeds the
 * tensor cores; codes and scales as b2a_gemm_q8 (rows x cols, cols a
 * multiple of 32), out [rows][ldo], 16-byte aligned, ldo a multiple of 8.
 * For a caller that keeps Q8_0 weights only and dequantizes each matrix into
 * one reusable buffer just before its b2a_gemm (the dequantized values the
 * reference computes per block inside its chunk GEMM, cuda.py:287-422). */
int b2a_q8_dequant(const void* codes, long long ldq, const void* scales, long long lds,
                   void* out, long long ldo, int dtype, int rows, int cols, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2ATTN_H_ */
