/*
 * motif_b200.h — C ABI of the B200 (sm_100a) Motif decode hot path.
 *
 * Plain extern "C" entry points: raw device pointers, element counts, a
 * cudaStream_t passed as void*, and an int status return (MOTIF_OK on
 * success). No C++ or framework types cross this boundary, so the Python
 * package (ctypes), a Swift MotifKit layer or any C caller binds it the same
 * way. All kernels are asynchronous on the given stream; inputs are read-only
 * unless a parameter says otherwise.
 *
 * Each declaration cites the reference interface it replaces (paths relative
 * to the junhoyeo/mlx-motif project root). The reference's operator layer is
 * src/mlx_motif/kernels/__init__.py:21-50; its cache API is
 * src/mlx_motif/cache.py.
 *
 * Runtime lengths: every KV length / cache offset can be given either as a
 * host integer or as a device int32 pointer (non-NULL pointer wins). The
 * device form keeps the value out of the launch, so a captured CUDA graph
 * replays at every length (the reference passes the length as a runtime
 * kernel input for the same reason, attention.py:42-51).
 */
#ifndef MOTIF_B200_H
#define MOTIF_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOTIF_API __attribute__((visibility("default")))
#else
#define MOTIF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MOTIF_OK 0
#define MOTIF_ERR_NULL 1          /* a required pointer is NULL            */
#define MOTIF_ERR_BAD_SHAPE 2     /* shapes inconsistent / out of range    */
#define MOTIF_ERR_BAD_CONTRACT 3  /* shape outside the kernel contract     */
#define MOTIF_ERR_DTYPE 4         /* dtype / bits not supported            */
#define MOTIF_ERR_CUDA 5          /* a CUDA runtime call failed            */
#define MOTIF_ERR_WORKSPACE 6     /* workspace missing or too small        */

/* ---- element types ----------------------------------------------------- */
#define MOTIF_F16 0
#define MOTIF_BF16 1
#define MOTIF_F32 2

/* Human-readable name of a status code. */
MOTIF_API const char* motif_status_string(int status);
/* Detail message of the last failed call on this host thread ("" if none). */
MOTIF_API const char* motif_last_error(void);
/* ABI version (bumped on any signature change). */
MOTIF_API int motif_abi_version(void);

/* ---- 4-slot KV cache view ------------------------------------------------
 * The four slots k1, k2, v1, v2 of one layer (cache.py:303-545), each
 * (batch, heads, capacity, head_dim) row-contiguous. bits == 16: data[i] are
 * fp16/bf16 rows. bits == 4 or 8: data[i] are packed uint32
 * (…, head_dim*bits/32) and scales[i]/biases[i] are (…, head_dim/group_size)
 * in the activation dtype (the MLX affine triple, cache.py:430-436). */
typedef struct motif_kv4_slots {
  void* data[4];
  void* scales[4];
  void* biases[4];
  int32_t bits;
  int32_t group_size;
  int64_t batch;
  int64_t heads;
  int64_t capacity;
  int64_t head_dim;
} motif_kv4_slots;

/* ---- PolyNorm -------------------------------------------------------------
 * y = w0*x^3/rms(x^3) + w1*x^2/rms(x^2) + w2*x/rms(x) + b over the last axis.
 * Replaces mlx_motif.kernels.polynorm (src/mlx_motif/kernels/mlp.py:119-157).
 * x, y: (rows, dim); weight (3,), bias (1,) in dtype. */
MOTIF_API int motif_polynorm(int dtype, const void* x, const void* weight, const void* bias, float eps,
                   int64_t rows, int64_t dim, void* y, void* stream);

/* act = polynorm(gate) * up, the MLP activation of MotifMLP.__call__
 * (src/mlx_motif/model.py:267-268). gate/up rows are `in_stride` elements
 * apart (so a fused [gate | up] GEMV output can be passed as two views). */
MOTIF_API int motif_polynorm_mul(int dtype, const void* gate, const void* up, int64_t in_stride,
                       const void* weight, const void* bias, float eps, int64_t rows, int64_t dim,
                       void* y, void* stream);

/* motif_polynorm_mul with the intermediate axis sharded over tensor-parallel
 * ranks: motif_polynorm_row_stats writes this rank's (Σx², Σx⁴, Σx⁶) of each
 * row's `dim` gate values to stats (rows × 3 fp32); once the caller has summed
 * them over the ranks, motif_polynorm_mul_stats applies PolyNorm·up to this
 * rank's slice with the means taken over full_dim values. No reference
 * counterpart (the reference is single-device); the arithmetic is
 * motif_polynorm_mul's (mlp.py:119-157, model.py:267-268). */
MOTIF_API int motif_polynorm_row_stats(int dtype, const void* x, int64_t in_stride, int64_t rows, int64_t dim,
                                       float* stats, void* stream);
MOTIF_API int motif_polynorm_mul_stats(int dtype, const void* gate, const void* up, int64_t in_stride,
                                       const void* weight, const void* bias, float eps, int64_t rows,
                                       int64_t dim, const float* stats, int64_t full_dim, void* y, void* stream);

/* ---- GDA post reduction -----------------------------------------------------
 * y = (o − λ·n[h/gr]) · rsqrt(mean(d²) + eps) · subln_w · (1 − λ_init).
 * Replaces gda_post_split (src/mlx_motif/kernels/gda.py:223-282).
 * attn_o (B, q_groups*gr, S, C), attn_n (B, q_groups, S, C), subln_w (C,) in
 * dtype; lambda_full fp32 device array of lambda_len ∈ {1, q_groups,
 * q_groups*gr} values (1 = the reference's per-layer scalar). */
MOTIF_API int motif_gda_post_split(int dtype, const void* attn_o, const void* attn_n, const void* subln_w,
                         const float* lambda_full, int64_t lambda_len, float lambda_init,
                         int64_t batch, int64_t q_groups, int64_t gr, int64_t seq, int64_t channels,
                         float eps, void* y, void* stream);

/* Same on the concatenated (origin | noise) input merged (B, q_groups*(gr+1), S, C).
 * Replaces gda_post (src/mlx_motif/kernels/gda.py:285-341). */
MOTIF_API int motif_gda_post(int dtype, const void* merged, const void* subln_w, const float* lambda_full,
                   int64_t lambda_len, float lambda_init, int64_t batch, int64_t q_groups,
                   int64_t gr, int64_t seq, int64_t channels, float eps, void* y, void* stream);

/* ---- shared-QK dual-V decode attention ------------------------------------
 * y = cat[softmax(q kᵀ·scale)·v1, softmax(q kᵀ·scale)·v2] with GQA broadcast
 * (q head h reads kv head h / (h_q/h_kv)); rows ≥ kv_len are never read.
 * Replaces sdpa_dual_v (src/mlx_motif/kernels/attention.py:190-260).
 * q (B, h_q, 1, D); k, v1, v2 (B, h_kv, kv_cap, D); y (B, h_q, 1, 2D).
 * Split-KV: the workspace holds per-split partials; pass workspace_bytes = 0
 * for a single split (no workspace). */
MOTIF_API size_t motif_sdpa_dual_v_workspace_bytes(int64_t batch, int64_t h_q, int64_t head_dim,
                                         int64_t max_splits);
MOTIF_API int motif_sdpa_dual_v(int dtype, const void* q, const void* k, const void* v1, const void* v2,
                      float scale, int64_t batch, int64_t h_q, int64_t h_kv, int64_t kv_cap,
                      int64_t head_dim, int64_t kv_len, const int32_t* kv_len_dev, void* y,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of motif_sdpa_dual_v, for callers that cannot call
 * cudaMalloc (a plugin whose device memory belongs to its host framework's
 * allocator, hot paths that must not take cudaMalloc's device-wide
 * synchronisation). It has no
 * counterpart in the reference. Its split-KV partials live in one
 * file-scope __device__ array of motif_sdpa_dual_v_static_scratch_bytes()
 * (4 MiB) that each GPU loading the library keeps until exit. The first
 * call on a device resolves the array's device address (concurrent first
 * calls from several host threads are safe). Shapes whose two-split partials
 * (batch*h_q*(2*head_dim+2)*4*2 bytes) exceed the array are rejected with
 * MOTIF_ERR_WORKSPACE. The rejection is deliberate: this entry is the
 * split-KV kernel with its partials in the array, and a shape too large for
 * it is refused with a clear error rather than silently run as one long
 * split (motif_sdpa_dual_v with workspace_bytes 0 is that one-split form,
 * for a caller that wants it). Nothing in the array needs to start at zero
 * (every split writes its partial before the merge reads it), but all calls
 * on one device share that device's copy: calls that overlap on the GPU
 * (on different streams) race and must be serialised by the caller. Otherwise
 * the same arguments and results as motif_sdpa_dual_v. */
MOTIF_API size_t motif_sdpa_dual_v_static_scratch_bytes(void);
MOTIF_API int motif_sdpa_dual_v_static(int dtype, const void* q, const void* k, const void* v1,
                                       const void* v2, float scale, int64_t batch, int64_t h_q,
                                       int64_t h_kv, int64_t kv_cap, int64_t head_dim, int64_t kv_len,
                                       const int32_t* kv_len_dev, void* y, void* stream);

/* Same attention reading MLX affine-quantized K, V1, V2 triples directly
 * (bits 4 or 8). Replaces sdpa_dual_v_q4 (attention.py:510-645) with the same
 * shape contract (attention.py:556-608): D % 32 == 0, D % group_size == 0,
 * (32/bits) % (D/32) == 0 and group_size % (D/32) == 0. */
MOTIF_API int motif_sdpa_dual_v_q(int dtype, int bits, int group_size, const void* q,
                        const uint32_t* k_data, const void* k_scales, const void* k_biases,
                        const uint32_t* v1_data, const void* v1_scales, const void* v1_biases,
                        const uint32_t* v2_data, const void* v2_scales, const void* v2_biases,
                        float scale, int64_t batch, int64_t h_q, int64_t h_kv, int64_t kv_cap,
                        int64_t head_dim, int64_t kv_len, const int32_t* kv_len_dev, void* y,
                        void* workspace, size_t workspace_bytes, void* stream);

/* One GDA decode layer's attention block in one pass over the 4-slot cache:
 * both sdpa_dual_v calls of MotifAttention._forward_grouped (model.py:716-768;
 * origin heads with k1, noise heads with k2, shared v1/v2) plus
 * gda_post_split, reading every cache row once. fp16 only, batch 1.
 * q: (q_groups*(gr+1), D) origin-first; out: (q_groups*gr, 2D) — the o_proj
 * input. cache->bits selects fp16 rows (16) or packed q4/q8. */
MOTIF_API size_t motif_gda_decode_attention_workspace_bytes(int64_t q_heads, int64_t head_dim,
                                                  int64_t max_splits);
MOTIF_API int motif_gda_decode_attention(const void* q, const motif_kv4_slots* cache, float scale,
                               int64_t q_groups, int64_t gr, int64_t kv_len,
                               const int32_t* kv_len_dev, const void* subln_w,
                               const float* lambda_full, int64_t lambda_len, float lambda_init,
                               float eps, void* out, void* workspace, size_t workspace_bytes,
                               void* stream);

/* The decoder's whole attention step for one layer in ONE launch:
 * motif_rope_qkv_append followed by motif_gda_decode_attention (reference
 * model.py:580-657 and 716-768: RoPE of q/k, the 4-slot cache write, both
 * sdpa_dual_v calls and gda_post_split). qkv: the fused projection row
 * [q heads | k1,k2 pairs | v1,v2 pairs] (fp16); pos_len: device int32
 * [pos, kv_len] — the new k/v row is written at pos and the attention covers
 * positions [0, kv_len). Results equal the two-call sequence bit for bit.
 * workspace: motif_gda_decode_step_workspace_bytes(q_heads, 128, splits)
 * bytes (splits <= 64), zero-filled before first use; its first 256 bytes
 * hold per-group counters that the kernel leaves zeroed.
 * Launched with programmatic dependent launch: before it waits for the
 * previous kernel in the stream it already reads pos_len, inv_freq and the
 * cache rows other than pos, so that previous kernel must not write those
 * (in the decoder it is the qkv projection). */
MOTIF_API size_t motif_gda_decode_step_workspace_bytes(int64_t q_heads, int64_t head_dim, int64_t max_splits);
MOTIF_API int motif_gda_decode_step(const void* qkv, const float* inv_freq, const motif_kv4_slots* cache,
                                    const int32_t* pos_len, float scale, int64_t q_groups, int64_t gr,
                                    const void* subln_w, const float* lambda_full, int64_t lambda_len,
                                    float lambda_init, float eps, void* out, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* The vanilla (ungrouped differential) decoder's attention step for one layer
 * in ONE launch: MotifAttention._forward_vanilla (reference model.py:486-559)
 * for batch 1, fp16. qkv: the fused projection row [q (2*H heads, q1/q2
 * interleaved) | k (2*kv_heads, k1/k2 interleaved) | v (2*kv_heads, the
 * projection's paired order v0_a, v0_b, v1_a, ...)], H = kv_heads*n_rep.
 * The cache is the 4-slot layout with kv_heads heads per slot: k1, k2, the
 * slab halves va and vb (cache.py:55-69). The new row is roped, written at
 * pos_len[0], and the step attends over [0, pos_len[1]): q1 heads score on
 * k1, q2 heads on k2, each against [va | vb]; then (o1 - lambda*o2), SubLN
 * over 2*head_dim and the (1 - lambda_init) scale, with MLX's fp16 rounding
 * at each op. out: (H, 2*head_dim) — the o_proj input. n_rep in {1, 2, 4},
 * head_dim 128, lambda_full one value. workspace: as motif_gda_decode_step's
 * with q_heads = 2*H; the same programmatic-dependent-launch precondition. */
MOTIF_API int motif_vanilla_decode_step(const void* qkv, const float* inv_freq, const motif_kv4_slots* cache,
                                        const int32_t* pos_len, float scale, int64_t kv_heads, int64_t n_rep,
                                        const void* subln_w, const float* lambda_full, float lambda_init,
                                        float eps, void* out, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* Which kernel motif_gda_decode_step / motif_vanilla_decode_step launch for
 * this cache (no reference counterpart: the reference has one Metal kernel
 * per dtype, kernels/attention.py:190-260 and 510-645). Returns
 * MOTIF_ATTN_KERNEL_TCGEN05 for the tensor-core long-cache step (fp16 rows,
 * or q4 group 64 with a capacity that is a multiple of 4, capacity at least
 * MOTIF_LONG_ATTN_MIN_CAP rows, default 2048, 16-byte aligned slots),
 * MOTIF_ATTN_KERNEL_SPLIT for the CUDA-core split-KV step, or a negative
 * status for a cache neither accepts. Pure host arithmetic on the view: no
 * CUDA call, so it answers on a machine without a GPU. */
#define MOTIF_ATTN_KERNEL_SPLIT 1
#define MOTIF_ATTN_KERNEL_TCGEN05 2
MOTIF_API int motif_decode_step_kernel(const motif_kv4_slots* cache);

/* ---- affine quantization ---------------------------------------------------
 * MLX-layout affine group quantization along the last axis (bits 4 or 8):
 * data (rows, dim*bits/32) uint32 little-endian, scales/biases
 * (rows, dim/group_size) in dtype. Replaces the mx.quantize call sites of the
 * cache (cache.py:399-402, 498). */
MOTIF_API int motif_quantize(int dtype, int bits, int group_size, const void* x, int64_t rows, int64_t dim,
                   uint32_t* data, void* scales, void* biases, void* stream);
/* Inverse, element ch = scale[g]*((data[ch/EL] >> (ch%EL)*bits) & mask) + bias[g].
 * Replaces _dequant_probe / mx.dequantize (src/mlx_motif/kernels/mlp.py:213-255). */
MOTIF_API int motif_dequantize(int dtype, int bits, int group_size, const uint32_t* data,
                     const void* scales, const void* biases, int64_t rows, int64_t dim, void* y,
                     void* stream);

/* ---- 4-slot cache writes ---------------------------------------------------
 * Write k1, k2, v1, v2 (B, heads, seq, D) at rows [offset, offset+seq) of the
 * slots (fp16 copy, or one batched quantize for bits 4/8). Replaces
 * MotifGroupedKVCache.update_and_fetch_4 (cache.py:337-360) and
 * MotifGroupedQuantizedKVCache._update_4 (cache.py:485-512); the caller owns
 * capacity and the offset bookkeeping. */
MOTIF_API int motif_kv4_append(int dtype, const motif_kv4_slots* cache, const void* k1, const void* k2,
                     const void* v1, const void* v2, int64_t seq, int64_t offset,
                     const int32_t* offset_dev, void* stream);

/* Decode prologue of _forward_grouped (model.py:580-657) for batch 1, S = 1:
 * split the fused qkv row (q_heads + 2*kv2 + 2*kv2 heads of D, Q origin-first,
 * k/v heads interleaved slot-1/slot-2), apply non-traditional RoPE at position
 * *pos_dev to q and k, write q to q_out (q_heads, D) and append k1, k2, v1,
 * v2 at row *pos_dev of the cache. inv_freq: fp32 (D/2,). fp16 only. */
MOTIF_API int motif_rope_qkv_append(const void* qkv, const float* inv_freq, int64_t q_heads,
                          const motif_kv4_slots* cache, const int32_t* pos_dev, void* q_out,
                          void* stream);

/* The same for a block of `seq` prompt rows: qkv (seq, q_heads + 4*kv2 heads
 * of 128), row s at position offset + s (offset = *offset_dev when
 * offset_dev is non-NULL); q is written head-major, q_out (q_heads, seq, 128)
 * (the layout motif_prefill_attention reads); k/v rows go to cache rows
 * [offset, offset + seq), quantized per row for a q4/q8 cache (bit-identical
 * to appending the rows one by one). Reference: the prompt branch of
 * _forward_grouped / _forward_vanilla (model.py:580-657, 486-521). */
MOTIF_API int motif_rope_qkv_append_rows(const void* qkv, int64_t seq, const float* inv_freq, int64_t q_heads,
                                         const motif_kv4_slots* cache, int64_t offset, const int32_t* offset_dev,
                                         void* q_out, void* stream);

/* Non-traditional RoPE on x (B, H, S, D) at positions offset + s (mlx-lm
 * initialize_rope, traditional=False, as used at model.py:414-420,589-594). */
MOTIF_API int motif_rope(int dtype, const void* x, int64_t batch, int64_t heads, int64_t seq, int64_t dim,
               int64_t offset, const int32_t* offset_dev, const float* inv_freq, void* y,
               void* stream);

/* ---- quantized linear ------------------------------------------------------
 * y (m, n) = x (m, k) · dequant(W)ᵀ with W in the nn.QuantizedLinear layout:
 * w (n, k*bits/32) uint32, scales/biases (n, k/group_size) in dtype. Replaces
 * mx.quantized_matmul behind nn.QuantizedLinear (every linear of the decoder,
 * model.py:437-442, 262-264, 894; fused qkv 1017-1079). Fast path: bits 4,
 * group 64, fp16, k % 128 == 0 (persistent stream-K GEMV; rows of x run one
 * after another); m >= 128 rows with n % 128 == 0 and k % 512 == 0 take the
 * tensor-core GEMM (motif_q4_gemm); other bits/groups/dtypes take a
 * CUDA-core path. The
 * workspace (motif_quantized_linear_workspace_bytes) must be zero-filled
 * before its first use; the kernel leaves it zeroed. Rows of a tile split
 * between warps are reduced by the tile's first warp, which waits for the
 * others' partials: the one-row GEMV's grid is at most one CTA per SM and
 * relies on all of them becoming resident (a wait that runs out after 200 ms
 * sets the workspace's error word). */
MOTIF_API size_t motif_quantized_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int bits,
                                              int group_size);
MOTIF_API int motif_quantized_linear(int dtype, int bits, int group_size, const void* x, int64_t m,
                           int64_t k, const uint32_t* w, const void* scales, const void* biases,
                           int64_t n, void* y, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Prompt-length q4 linear on the tcgen05 tensor cores: y (m, n) = x (m, k) ·
 * dequant(W)ᵀ [+ residual], fp16 x / y / residual row-major, W q4 group 64 in
 * the nn.QuantizedLinear layout (reference: mx.quantized_matmul behind every
 * nn.QuantizedLinear of a prompt forward, model.py:1047-1079). Weight tiles
 * are dequantized to fp16 in shared memory and multiplied with fp32
 * accumulation in tensor memory; y is rounded to fp16 once, then (with
 * residual) added in fp16 like the reference's h + linear(x). Needs
 * m >= 128, n % 128 == 0, k % 512 == 0 and 16-byte aligned operands. err
 * (optional, device int): set to 1 if a pipeline wait timed out. */
MOTIF_API int motif_q4_gemm(const void* x, int64_t m, int64_t k, const uint32_t* w, const void* scales,
                            const void* biases, int64_t n, void* y, const void* residual, int* err,
                            void* stream);

/* ---- prompt (prefill) attention -------------------------------------------
 * Causal attention of `seq` prompt rows at positions [offset, offset + seq)
 * over cache rows [0, offset + seq) of an fp16 4-slot cache (the rows already
 * appended), on the tcgen05 tensor cores with fp32 accumulation. Per query
 * head: o = softmax(q·kᵀ·scale, causal)·[v1 | v2] (256 wide), with
 *   mode 0 (grouped): q_heads = kv2*(gr+1) origin-first; origin head h reads
 *     k1 of group h/gr, noise head q_origin+g reads k2 of group g — the four
 *     per-slab SDPAs of _forward_grouped's prompt path (model.py:769-807);
 *   mode 1 (vanilla): q_heads = 2*kv2*gr (gr = n_rep), q1/q2 interleaved;
 *     head h reads k1 (even h) or k2 (odd h) of kv head (h/2)/gr — the
 *     per-slab SDPAs of _forward_vanilla (model.py:486-559).
 * q: head-major (q_heads, seq, 128) fp16; out: (seq, q_heads, 256) fp16, each
 * SDPA output rounded to fp16 as the reference's are. err (optional device
 * int) is set to 1 if a pipeline wait timed out. */
MOTIF_API int motif_prefill_attention(const void* q, int64_t seq, int64_t q_heads, const motif_kv4_slots* cache,
                                      int64_t offset, int mode, int64_t gr, float scale, void* out, int* err,
                                      void* stream);

/* motif_prefill_attention for a short block over a long cache (the [1, K+1]
 * speculative verify, prompt tails): with seq <= 128 and a workspace of at least
 * motif_prefill_attention_split_workspace_bytes(seq, q_heads) bytes, the cache
 * rows are divided among up to 16 CTAs per query head (at least two 64-row
 * tiles each at `offset`, at most one CTA per SM in total) whose fp32 softmax
 * states a second kernel merges; otherwise it is motif_prefill_attention.
 * Results agree with it within fp32 rounding before the fp16 output.
 * offset_dev (optional device int32): the position of query 0 is read there at
 * run time (a CUDA graph replayed at every offset); `offset` is then the
 * largest value it may hold, used for the launch shape, and splits left
 * without key tiles at a smaller offset contribute nothing. A device offset
 * outside [0, capacity - seq] sets *err and reads nothing. No reference
 * counterpart beyond motif_prefill_attention's (the same SDPAs, model.py:486-559,
 * 769-807). */
MOTIF_API size_t motif_prefill_attention_split_workspace_bytes(int64_t seq, int64_t q_heads);
MOTIF_API int motif_prefill_attention_split(const void* q, int64_t seq, int64_t q_heads,
                                            const motif_kv4_slots* cache, int64_t offset, const int32_t* offset_dev,
                                            int mode, int64_t gr, float scale, void* out, void* workspace,
                                            size_t workspace_bytes, int* err, void* stream);

/* The differential combine over prompt rows: o (seq, q_heads, 256) from
 * motif_prefill_attention -> y (seq, out_heads, 256), the o_proj input.
 * mode 0: gda_post_split (kernels/gda.py:223-282) of each group's gr origin
 * heads against its noise head; lambda_len 1, groups or groups*gr.
 * mode 1: the vanilla (o1 - lambda*o2), SubLN, (1 - lambda_init) of each
 * q1/q2 pair with fp16 rounding after each op (model.py:553-557);
 * lambda_len 1. */
MOTIF_API int motif_prefill_post(const void* o, int64_t seq, int64_t q_heads, int mode, int64_t groups, int64_t gr,
                                 const void* subln_w, const float* lambda_full, int64_t lambda_len,
                                 float lambda_init, float eps, void* y, void* stream);

/* Fused decode linear: the q4 GEMV of motif_quantized_linear (bits 4, group 64,
 * fp16, one input row) with the input vector built in its prologue and an
 * optional statistics epilogue, so the decoder's norms and activations need no
 * kernels of their own. Replaces, per layer of MotifDecoderLayer
 * (model.py:845-855): input_layernorm + qkv_proj (mode 1), o_proj (mode 0),
 * residual + post_attention_layernorm + gate/up (mode 1 + stats), PolyNorm·up
 * + down_proj (mode 2, model.py:267-268); final norm + lm_head (mode 1,
 * model.py:879, 905).
 *   mode 0: x given.
 *   mode 1: v = (token ? embed[*token] : h_in) + delta (delta may be NULL, the
 *           sum rounded to fp16 as the reference's residual add); x =
 *           rms_norm(v)·norm_w (eps); v is written to h_out when non-NULL
 *           (h_out must not alias h_in).
 *   mode 2: x = fp16(polynorm(gate))·up, PolyNorm statistics = the sum of
 *           stats_count (Σg², Σg⁴, Σg⁶) triplets at `stats`, mean over poly_dim.
 * argmax_out (optional): the greedy token — index of the largest fp16 output
 * (first on ties, NaN below everything, as motif_argmax) — written once the
 * last output tile is done; the lm_head then needs no argmax launch (greedy
 * sampling in mlx-lm generate_step). pos_len_inc (optional, with argmax_out):
 * int32[2] incremented by one each after the token is written (the decode
 * step's position and kv_len). This state lives in the workspace's counter
 * region, so a workspace serves one such launch at a time.
 * argmax_key_out (optional, for a vocabulary shard of a tensor-parallel
 * lm_head): the winner as one int64 key — order-preserving value bits above
 * the inverted GLOBAL row (row + argmax_row_offset), top bit flipped — so the
 * largest key over all shards (an int64 MAX all-reduce) is the global greedy
 * token; motif_argmax_key_decode turns it into the token.
 * Tensor-parallel exchange (replaces the all-reduces of a row-parallel
 * o_proj / down_proj and of the PolyNorm statistics, reference model.py:836
 * and 267): a producer stores each fp32 output row (tp_out) and/or each tile
 * statistic (tp_stats) into every rank's buffer as a (value, number) pair —
 * one 8-byte store, so a pair is valid on its own and no fence or flag is
 * needed; a consumer reads the pairs of all ranks, re-reading (bounded) any
 * whose number is not yet this exchange's: tp_in in mode 1 (the residual delta
 * is the fp16-rounded sum of the ranks' partials, summed in rank order, so
 * every rank gets the same bits), tp_stats_in in mode 2. Buffers come from
 * motif_ipc_alloc / motif_ipc_open and must be zeroed whenever the position
 * is rewound. A wait that runs out sets the workspace's error word and the
 * kernel goes on (its outputs are then garbage).
 * stats_out (optional): for output rows [0, stats_rows) (a multiple of 16),
 * one (Σy², Σy⁴, Σy⁶) triplet per 16-row tile of the fp16-rounded outputs.
 * workspace: motif_linear_fused_workspace_bytes(n, k) bytes, zero-filled
 * before first use (the kernel leaves it zeroed; split tiles are reduced as in
 * motif_quantized_linear). Its first 64 KiB
 * hold per-tile counters at a fixed place, so one workspace sized for the
 * largest shape serves GEMVs of every shape in turn; launched with programmatic
 * stream serialization, it starts streaming weights while the previous kernel
 * finishes. Before it waits for that kernel it also reads the weights and the
 * prologue's constants (norm_w, poly_w, poly_b), so the previous kernel in the
 * stream must not write those. With a tensor-parallel exchange, CTA 0 adds the
 * nanoseconds its exchange reads took (waits for the peers included) to the
 * int64 at byte 65504 of the workspace; the caller reads and zeroes it. */
typedef struct motif_linear_io {
  int32_t mode;
  const void* x;
  const void* h_in;
  const int32_t* token;
  const void* embed;
  int64_t vocab;
  const void* delta;
  void* h_out;
  const void* norm_w;
  float eps;
  const void* gate;
  const void* up;
  const float* stats;
  int64_t stats_count;
  const void* poly_w;
  const void* poly_b;
  float poly_eps;
  int64_t poly_dim;
  float* stats_out;
  int64_t stats_rows;
  int32_t* argmax_out;
  int32_t* pos_len_inc;
  int64_t* argmax_key_out;
  int64_t argmax_row_offset;
  /* tensor-parallel exchange over peer memory (optional; tp_world <= 8). Every
   * value travels as one 8-byte (fp32 value, int32 number) pair, number =
   * (*tp_seq + 1) * 1024 + tp_tag. */
  int32_t tp_world;
  const int32_t* tp_seq;        /* device int32 (the decode position) */
  int32_t tp_tag;               /* 0..1023: which exchange of the step */
  int64_t* tp_out[8];           /* producer: this rank's output rows' pairs in each rank's buffer */
  int64_t* tp_stats[8];         /* producer: this rank's tile statistics' pairs in each rank's buffer */
  const int64_t* tp_in;         /* consumer, mode 1: [tp_world][K] pairs; delta = fp16(sum of the ranks') */
  const int64_t* tp_stats_in;   /* consumer, mode 2: [stats_count][3] pairs of all ranks' tiles */
} motif_linear_io;

MOTIF_API size_t motif_linear_fused_workspace_bytes(int64_t n, int64_t k);
MOTIF_API int motif_linear_fused(const motif_linear_io* io, const uint32_t* w, const void* scales,
                                 const void* biases, int64_t n, int64_t k, void* y, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ---- peer-to-peer buffers for the tensor-parallel exchange --------------------
 * No reference counterpart (the reference runs on one device). One buffer per
 * rank from cudaMalloc, shared with the other processes of the node through
 * CUDA IPC: motif_ipc_alloc returns the pointer and a handle of
 * motif_ipc_handle_bytes() bytes; the other ranks motif_ipc_open that handle.
 * The buffer is zero-filled. */
MOTIF_API size_t motif_ipc_handle_bytes(void);
MOTIF_API int motif_ipc_alloc(size_t bytes, void** ptr, void* handle);
MOTIF_API int motif_ipc_open(const void* handle, void** ptr);
MOTIF_API int motif_ipc_close(void* ptr);
MOTIF_API int motif_ipc_zero(void* ptr, size_t bytes, void* stream);
MOTIF_API int motif_ipc_free(void* ptr);

/* ---- decoder glue (model.py:845-905) ---------------------------------------- */
/* y = rms_norm(x) * w (nn.RMSNorm, model.py:850-851, 864). */
MOTIF_API int motif_rms_norm(int dtype, const void* x, const void* w, float eps, int64_t rows, int64_t dim,
                   void* y, void* stream);
/* h += delta (residual, model.py:854-855), then y = rms_norm(h) * w. h is in/out. */
MOTIF_API int motif_add_rms_norm(int dtype, void* h, const void* delta, const void* w, float eps,
                       int64_t rows, int64_t dim, void* y, void* stream);
/* h = table[*token_dev] (nn.Embedding, model.py:862/872), y = rms_norm(h) * w. */
MOTIF_API int motif_embed_rms_norm(int dtype, const int32_t* token_dev, const void* table, int64_t vocab,
                         int64_t dim, const void* w, float eps, void* h, void* y, void* stream);
/* The same for a block of prompt rows: h (rows, dim) = table[tokens_dev[r]],
 * y = rms_norm(h) * w (the prompt forward's embedding and first input norm). */
MOTIF_API int motif_embed_rms_norm_rows(int dtype, const int32_t* tokens_dev, int64_t rows, const void* table,
                                        int64_t vocab, int64_t dim, const void* w, float eps, void* h, void* y,
                                        void* stream);
/* ---- sampling ------------------------------------------------------------
 * Temperature sampling of `rows` logit rows (fp16, row_stride apart) by the
 * Gumbel-max rule — token = argmax(l/T + g), g = -log(-log u), u from
 * Philox-4x32-10 keyed by `seed` and counted by (element, position, row,
 * stream_id) — which draws exactly from softmax(l/T) (top-p 1.0). T = 0 is the
 * greedy argmax. position = *pos_dev when given (a replayed graph draws fresh
 * numbers at every position), else pos_host. pos_len_inc (optional int32[2])
 * is advanced by one after row 0, as the decode step's head does. Reference:
 * mlx-lm generate_step's categorical sampler at temperature T. */
MOTIF_API int motif_sample(const void* logits, int64_t rows, int64_t n, int64_t row_stride, float temperature,
                           uint64_t seed, const int32_t* pos_dev, int64_t pos_host, uint32_t stream_id,
                           int32_t* tokens, void* pos_len_inc, void* stream);

/* motif_sample for one shard of a vocabulary split over tensor-parallel ranks
 * (no reference counterpart: the reference samples on one device through
 * mlx-lm's generate_step). logits: this rank's n values, global vocabulary
 * indices row_offset .. row_offset + n - 1; the Gumbel noise is drawn for the
 * global index, so the ranks together draw exactly what motif_sample draws for
 * the whole row. key_out (int64, device): the largest order-preserving key of
 * l/T + g in the shard as a signed value; an int64 MAX all-reduce of the ranks'
 * keys followed by motif_argmax_key_decode yields the token. */
MOTIF_API int motif_sample_key(const void* logits, int64_t n, float temperature, uint64_t seed,
                               const int32_t* pos_dev, int64_t pos_host, uint32_t stream_id, int64_t row_offset,
                               int64_t* key_out, void* stream);

/* Speculative acceptance of k draft tokens (rejection sampling, the reference's
 * MotifSpeculativeDecoding): p_logits are the target's k+1 rows (positions of
 * the draft tokens and the bonus position), q_logits the draft's k rows, both
 * fp16 with row_stride. Draft token i is accepted with probability
 * min(1, p_i(x_i)/q_i(x_i)); at the first rejection the next token is drawn
 * from max(0, p_i - q_i) renormalised, after k acceptances from p_k. T = 0:
 * accept while the draft equals the target's argmax, next token = that row's
 * argmax (q_logits may be NULL). out: int32[2] = {accepted, next token}. */
MOTIF_API int motif_speculative_accept(const void* p_logits, const void* q_logits, int64_t row_stride,
                                       const int32_t* draft_tokens, int64_t k, int64_t n, float temperature,
                                       uint64_t seed, const int32_t* pos_dev, int64_t pos_host, int32_t* out,
                                       void* stream);

/* Greedy sampler: first index of the maximum of logits (n,) -> *out_index
 * (argmax at temperature 0 in mlx_lm generate_step). */
MOTIF_API size_t motif_argmax_workspace_bytes(int64_t n);
/* Token (and optional pos_len int32[2] += 1) from a key of argmax_key_out,
 * after the shards' keys were combined with an int64 MAX all-reduce. */
MOTIF_API int motif_argmax_key_decode(const int64_t* key, int32_t* token, int32_t* pos_len_inc, void* stream);
/* The same token without a collective: the ranks' keys meet over peer memory (no reference
 * counterpart: the reference is single-device). key: this rank's key (argmax_key_out or
 * motif_sample_key). slots (host array of `world` device pointers): each rank's key area of
 * 2*world int64 in its peer-visible buffer (motif_ipc_alloc / motif_ipc_open), zeroed whenever
 * the position is rewound. One launch tags the key with the step read from pos_dev[0], stores it
 * into slot [(pos & 1) * world + rank] of every rank's area, waits (at most 2 s, then err = 2)
 * until its own area holds all ranks' keys of this step, writes the token of the largest and
 * advances pos_len_inc. Global rows must be below 2^24 - 1. Every rank launches it once per
 * step, in the same step order. */
MOTIF_API int motif_argmax_key_exchange(const int64_t* key, int64_t* const* slots, int world, int rank,
                                        const int32_t* pos_dev, int32_t* token, int32_t* pos_len_inc,
                                        int32_t* err, void* stream);
MOTIF_API int motif_argmax(int dtype, const void* logits, int64_t n, int32_t* out_index, void* workspace,
                 size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOTIF_B200_H */
