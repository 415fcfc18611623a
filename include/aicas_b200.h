/*
 * aicas_b200.h — C ABI of the B200 (sm_100a) attention backend for the
 * Qwen3-VL-2B inference hot path.
 *
 * Every entry point takes plain pointers, sizes and element strides, launches
 * on the caller's stream, allocates nothing, never synchronises the device and
 * returns an int status (AICAS_OK on success).  The exceptions are the one-time
 * set-up calls of the cross-GPU exchange (aicas_peer_buffer_*) and the health
 * query aicas_device_error_flags.  On failure a message is kept in
 * a thread-local buffer readable through aicas_last_error().
 *
 * The entry points replace these operators of the reference package
 * `triton_qwen3vl` (paths relative to the reference project):
 *
 *   aicas_decode_gqa          triton_qwen3vl/gqa_decode_attention.py:268-327
 *                             (_gqa_decode_attention_forward: q_len == 1 GQA
 *                             decode returning out and a base-2 LSE), extended
 *                             with a per-request length vector and split-KV
 *   aicas_merge_partials      no single reference line: the (out, LSE) merge the
 *                             reference never needed because it has no split-KV;
 *                             it combines partials produced by aicas_decode_gqa
 *                             on several devices (sequence-sharded caches)
 *   aicas_exchange_merge      no reference counterpart (single-device reference):
 *                             the same merge, with the partials moved between
 *                             the GPUs over NVLink peer memory in the same kernel
 *   aicas_prefill_gqa_causal  triton_qwen3vl/gqa_flash_attention.py:193-251
 *                             (_gqa_flash_attention_forward, causal, q_len == kv_len)
 *   aicas_varlen_attention    triton_qwen3vl/varlen_flash_attention.py:271-351
 *                             (_varlen_flash_attention_forward, non-causal,
 *                             packed sequences described by cu_seqlens)
 *   aicas_rope_kv_append      HF apply_rotary_pos_emb (transformers
 *                             models/qwen3_vl/modeling_qwen3_vl.py:410-432) followed by
 *                             the in-place cache write of
 *                             dujunbaoV1/evaluation_wrapper.py:84-100
 *                             (InplaceDecodeCacheLayer.update); optional per-head
 *                             RMSNorm as in dujunbaoV1/native_cuda_ops/
 *                             decode_q1_gqa_kernel.cu:376-480
 *   aicas_vision_rope         HF apply_rotary_pos_emb_vision (transformers
 *                             models/qwen3_vl/modeling_qwen3_vl.py:131-142) as the
 *                             vision attention applies it after splitting the
 *                             packed QKV projection (:205-209), in one kernel
 *   aicas_vision_qkv_rope     the vision attention's packed QKV projection (nn.Linear,
 *                             transformers models/qwen3_vl/modeling_qwen3_vl.py:205)
 *                             with the split and apply_rotary_pos_emb_vision (:206-209,
 *                             :131-142) in its epilogue, one kernel
 *   aicas_decode_linear       the decode-side matrix-vector products of
 *                             dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu:
 *                             rmsnorm_kernel :127-157 (as a fused prologue),
 *                             gate_up_silu_matvec_kernel :174-220 (SWIGLU),
 *                             dual_linear_matvec_kernel :222-269 and
 *                             qkv_linear_matvec_kernel :271-331 (segments),
 *                             lm_head_argmax_stage1/2 :482-575 (the LM-head
 *                             product; argmax stays with the caller), plus the
 *                             residual add of HF Qwen3VLTextDecoderLayer
 *                             (modeling_qwen3_vl.py:545-563)
 *
 * Layout conventions: attention tensors are 4-D [batch, heads, tokens, head_dim]
 * with head_dim contiguous (stride 1).  Strides are given in ELEMENTS.  All
 * device pointers must be 16-byte aligned and every stride times the element
 * size must be a multiple of 16 bytes.
 */
#ifndef AICAS_B200_H
#define AICAS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AICAS_API __attribute__((visibility("default")))
#else
#define AICAS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AICAS_ABI_VERSION 2

/* element types */
#define AICAS_DTYPE_F32 0
#define AICAS_DTYPE_F16 1
#define AICAS_DTYPE_BF16 2

/* status codes */
#define AICAS_OK 0
#define AICAS_ERR_INVALID 1     /* malformed argument (null pointer, bad stride, ...) */
#define AICAS_ERR_UNSUPPORTED 2 /* well-formed but outside what the kernels support */
#define AICAS_ERR_CUDA 3        /* a CUDA runtime call failed */
#define AICAS_ERR_WORKSPACE 4   /* workspace missing or too small */

/* bits of the device-side error word (see aicas_device_error_flags) */
#define AICAS_DEVERR_WAIT_TIMEOUT 1u /* a bounded barrier wait gave up */
#define AICAS_DEVERR_TMEM 2u         /* tensor-memory allocation returned an unusable address */
#define AICAS_DEVERR_PEER_TIMEOUT 4u /* a peer rank did not publish its partial in time */

/* ------------------------------------------------------------------------ */
/* GQA decode: one query token per request against that request's KV cache. */
/* ------------------------------------------------------------------------ */
typedef struct aicas_decode_params {
  const void* q;           /* [B, Hq, 1, D] */
  const void* k;           /* [B, Hkv, L, D]; consecutive tokens D elements apart */
  const void* v;           /* [B, Hkv, L, D]; consecutive tokens D elements apart */
  void* out;               /* [B, Hq, 1, D] same dtype as q; may be NULL if partial_o is set */
  float* lse;              /* optional [B, Hq] fp32, base-2 log-sum-exp of the scaled logits
                              (same convention as gqa_decode_attention.py:141) */
  float* partial_o;        /* optional [B, Hq, D] fp32 normalised output, for a cross-device
                              merge with aicas_merge_partials (lse must then be set too) */
  const int32_t* kv_lens;  /* optional [B] valid cache length per request (0..L); NULL = L */
  int64_t q_stride_b, q_stride_h;
  int64_t k_stride_b, k_stride_h;
  int64_t v_stride_b, v_stride_h;
  int64_t o_stride_b, o_stride_h; /* strides of out (ignored when out is NULL) */
  int32_t batch, num_q_heads, num_kv_heads, head_dim;
  int32_t kv_capacity;     /* L: allocated cache length, upper bound of kv_lens */
  int32_t dtype;           /* AICAS_DTYPE_* of q, k, v, out */
  float sm_scale;
  int32_t split_tokens;    /* tokens per split-KV work unit; 0 = choose automatically (for
                              many (request, KV head) pairs a halving table: the first split
                              of each cache the longest, later ones down to 1/8 of it) */
  const int32_t* kv_starts; /* optional [B] first valid cache slot per request; request b attends
                              to slots [kv_starts[b], kv_lens[b]) (a left-padded batch: the
                              slots before are padding); NULL = 0 */
} aicas_decode_params;

/* Bytes of device workspace aicas_decode_gqa needs for these parameters (0 when
   every request fits one split).  Layout: split counters in the first 1 MiB
   (one uint32 per (request, KV head), at most 262144 pairs), then fp32 partial
   outputs and LSEs.  Zero-fill the workspace once when it is allocated: every
   completed call leaves the counter region zeroed again, so one buffer can be
   reused by later calls of any shape on the same stream without clearing.
   Calls that may overlap on the device need separate workspaces.  After a
   device error (aicas_device_error_flags != 0) zero-fill it again. */
AICAS_API size_t aicas_decode_workspace_bytes(const aicas_decode_params* p);

AICAS_API int aicas_decode_gqa(const aicas_decode_params* p, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Same computation as aicas_decode_gqa, for callers that cannot allocate device
   memory: no counterpart in the reference.  Some hosts hand this library only
   the pointers of tensors they own and have no way to allocate more (their
   allocator is not exposed across the C boundary, or their device memory is
   reserved up front and cudaMalloc is not allowed); this entry point needs no
   workspace from them.  Its split-KV scratch is one static 8 MiB array inside
   the library (held by every GPU that loads it, until exit), enough for about
   7 MiB of partial results (B * Hkv * splits * G * (D + 1) * 4 bytes);
   larger requests are rejected with AICAS_ERR_UNSUPPORTED (raise split_tokens
   or use aicas_decode_gqa).  The first call in a CUDA context looks up the
   array's device address in that context and should come before any stream
   capture in it.
   Every call shares the one array and clears the counters it uses on
   `stream` before launching, so calls that may overlap on the device (other
   streams, other host threads) race and must be serialised by the caller. */
AICAS_API int aicas_decode_gqa_noalloc(const aicas_decode_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Merge P partial (out, LSE) pairs into the final output.                   */
/* ------------------------------------------------------------------------ */
typedef struct aicas_merge_params {
  const float* partial_o;   /* [P, B, H, D] fp32, contiguous */
  const float* partial_lse; /* [P, B, H] fp32 base-2 LSE, contiguous */
  void* out;                /* [B, H, D] (strided) */
  float* lse;               /* optional [B, H] merged LSE */
  int64_t o_stride_b, o_stride_h;
  int32_t num_partials, batch, num_heads, head_dim;
  int32_t dtype;            /* dtype of out */
} aicas_merge_params;

AICAS_API int aicas_merge_partials(const aicas_merge_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Cross-GPU merge of sequence-sharded decode partials over NVLink peer      */
/* memory.  No reference counterpart (the reference is single-device); it    */
/* replaces an all-gather of the partials followed by aicas_merge_partials.  */
/*                                                                          */
/* Set-up (once per process group, not on the hot path): every rank          */
/* allocates an exchange buffer of aicas_exchange_buffer_bytes() with         */
/* aicas_peer_buffer_alloc (the only entry points that allocate), shares the  */
/* 64-byte IPC handle with the other ranks, and maps theirs with              */
/* aicas_peer_buffer_open.  Each aicas_exchange_merge call is collective: all */
/* ranks make the same sequence of calls with the same sizes.  A rank waits   */
/* at most wait_budget_ns (default 4 s) for the others, then sets             */
/* AICAS_DEVERR_PEER_TIMEOUT, writes zeros and returns; the buffers are then  */
/* out of step and must be re-created.  One CTA per rank pushes to each      */
/* destination in parallel; launched with programmatic dependent launch, so  */
/* its launch overlaps the end of the decode kernel that produced the        */
/* partial.                                                                  */
/* ------------------------------------------------------------------------ */
#define AICAS_MAX_EXCHANGE_RANKS 8
#define AICAS_IPC_HANDLE_BYTES 64

AICAS_API size_t aicas_exchange_buffer_bytes(int32_t world, int32_t batch, int32_t num_heads, int32_t head_dim);
/* cudaMalloc'd, zeroed buffer of `bytes` on the current device and its IPC handle. */
AICAS_API int aicas_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
AICAS_API int aicas_peer_buffer_free(void* ptr);
/* Maps another rank's buffer (its IPC handle) into the current device. */
AICAS_API int aicas_peer_buffer_open(const void* ipc_handle, void** ptr);
AICAS_API int aicas_peer_buffer_close(void* ptr);

typedef struct aicas_exchange_params {
  void* peers[AICAS_MAX_EXCHANGE_RANKS]; /* rank r's buffer as mapped here (own buffer at [rank]) */
  const float* partial_o;   /* [B, H, D] fp32 local partial, contiguous */
  const float* partial_lse; /* [B, H] fp32 base-2 LSE, contiguous */
  void* out;                /* [B, H, D] (strided) merged output */
  float* lse;               /* optional [B, H] merged LSE */
  int64_t o_stride_b, o_stride_h;
  int32_t world, rank, batch, num_heads, head_dim;
  int32_t dtype;            /* dtype of out */
  uint64_t wait_budget_ns;  /* how long a rank waits for the others' partials before it gives up
                               (sets AICAS_DEVERR_PEER_TIMEOUT, writes zeros); 0 = 4 s */
} aicas_exchange_params;

AICAS_API int aicas_exchange_merge(const aicas_exchange_params* p, void* stream);

/* The sequence-sharded decode with the exchange fused into the decode kernel:
   every rank decodes its shard of every cache (p: out = the merged [B, Hq, 1, D]
   output, lse = the optional merged LSE, partial_o = NULL) and each (request,
   KV head) result goes straight into every rank's exchange buffer; a CTA whose
   own work is done merges pairs whose results have arrived from every rank.
   Replaces aicas_decode_gqa(partial_o) + aicas_exchange_merge (one launch, no
   partials in HBM).  The buffers are the exchange buffers of
   aicas_exchange_buffer_bytes(world, batch, num_q_heads, head_dim), shared with
   aicas_exchange_merge; 16-bit caches, head_dim 128.  Collective: every rank
   calls it in the same order.  The workspace (zero-initialised once, left zeroed
   by every call) is aicas_decode_exchange_workspace_bytes(p) bytes or more. */
typedef struct aicas_peer_group {
  void* peers[AICAS_MAX_EXCHANGE_RANKS]; /* rank r's exchange buffer as mapped here (own buffer at [rank]) */
  int32_t world, rank;
  uint64_t wait_budget_ns;  /* bound of the wait for the peers' results (sets AICAS_DEVERR_PEER_TIMEOUT,
                               writes zeros); 0 = 4 s */
} aicas_peer_group;

AICAS_API size_t aicas_decode_exchange_workspace_bytes(const aicas_decode_params* p);
AICAS_API int aicas_decode_gqa_exchange(const aicas_decode_params* p, const aicas_peer_group* group,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Flash attention on the tensor cores (tcgen05): causal GQA prefill and     */
/* non-causal packed-varlen attention.                                       */
/* ------------------------------------------------------------------------ */
typedef struct aicas_fmha_params {
  const void* q;            /* [B, Hq, Sq, D] */
  const void* k;            /* [B, Hkv, Skv, D] */
  const void* v;            /* [B, Hkv, Skv, D] */
  void* out;                /* [B, Hq, Sq, D] */
  int64_t q_stride_b, q_stride_h, q_stride_s;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  int64_t o_stride_b, o_stride_h, o_stride_s;
  int32_t batch, num_q_heads, num_kv_heads, seq_len_q, seq_len_kv, head_dim;
  int32_t dtype;            /* AICAS_DTYPE_F16 or AICAS_DTYPE_BF16 */
  float sm_scale;
  const int32_t* cu_seqlens_q; /* varlen only: [num_seqs + 1] int32 on the device */
  const int32_t* cu_seqlens_k; /* varlen only: [num_seqs + 1] int32 on the device */
  int32_t num_seqs;            /* varlen only */
  const int32_t* kv_starts;    /* causal prefill only, optional: [B] int32 on the device, the first
                                  valid position of each batch row (a left-padded batch); query row
                                  i of batch b attends to keys [kv_starts[b], i], rows before
                                  kv_starts[b] get zeros; NULL = 0 */
} aicas_fmha_params;

/* q_len == kv_len causal prefill, Hq a multiple of Hkv (gqa_flash_attention.py:12-46). */
AICAS_API int aicas_prefill_gqa_causal(const aicas_fmha_params* p, void* stream);

/* Block-diagonal non-causal attention over packed sequences, B == 1,
   Hq == Hkv (varlen_flash_attention.py:58-99).  Reads cu_seqlens on the device:
   no host synchronisation. */
AICAS_API int aicas_varlen_attention(const aicas_fmha_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused (optional q/k RMSNorm) + RoPE + KV-cache append.                    */
/* ------------------------------------------------------------------------ */
typedef struct aicas_rope_append_params {
  const void* q_in;         /* [B, Hq, S, D] */
  void* q_out;              /* [B, Hq, S, D] rotated q (may alias q_in) */
  const void* k_in;         /* [B, Hkv, S, D] new keys (before RoPE) */
  const void* v_in;         /* [B, Hkv, S, D] new values */
  const void* cos;          /* [B, S, D] */
  const void* sin;          /* [B, S, D] */
  void* k_cache;            /* [B, Hkv, C, D] */
  void* v_cache;            /* [B, Hkv, C, D] */
  const int32_t* positions; /* [B] slot of the first new token per request */
  int32_t* kv_lens_out;     /* optional [B]: receives min(positions[b] + S, C) */
  const void* q_norm_weight; /* optional [D] (dtype of q): per-head RMSNorm before RoPE */
  const void* k_norm_weight; /* optional [D] */
  float norm_eps;
  int64_t qi_stride_b, qi_stride_h, qi_stride_s;
  int64_t qo_stride_b, qo_stride_h, qo_stride_s;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  int64_t cs_stride_b, cs_stride_s;  /* strides of cos and sin (same for both) */
  int64_t kc_stride_b, kc_stride_h;  /* cache token stride is D */
  int64_t vc_stride_b, vc_stride_h;
  int32_t batch, num_q_heads, num_kv_heads, seq_len, head_dim, capacity;
  int32_t dtype;            /* dtype of q, k, v, caches and norm weights */
  int32_t cs_dtype;         /* dtype of cos/sin: same as dtype, or AICAS_DTYPE_F32 */
} aicas_rope_append_params;

AICAS_API int aicas_rope_kv_append(const aicas_rope_append_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Vision-tower RoPE of q and k (HF apply_rotary_pos_emb_vision), bit-exact.  */
/* ------------------------------------------------------------------------ */
typedef struct aicas_vision_rope_params {
  const void* q_in;         /* [T, H, D] (e.g. views into the packed qkv projection [T, 3, H, D]) */
  const void* k_in;
  void* q_out;              /* [T, H, D] rotated (may not alias the inputs) */
  void* k_out;
  const float* cos;         /* [T, D] fp32 */
  const float* sin;         /* [T, D] fp32 */
  int64_t qi_stride_t, qi_stride_h, ki_stride_t, ki_stride_h;
  int64_t qo_stride_t, qo_stride_h, ko_stride_t, ko_stride_h;
  int64_t cs_stride_t;      /* row stride of cos and sin */
  int32_t tokens, heads, head_dim; /* head_dim a multiple of 16 */
  int32_t dtype;            /* AICAS_DTYPE_F16 or AICAS_DTYPE_BF16 */
} aicas_vision_rope_params;

AICAS_API int aicas_vision_rope(const aicas_vision_rope_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Vision-tower packed QKV projection with the RoPE of q and k in its        */
/* epilogue, on the tensor cores: out = [q_rot | k_rot | v] of x W^T + b.    */
/* ------------------------------------------------------------------------ */
typedef struct aicas_vision_qkv_params {
  const void* x;            /* [T, K] patch features, x_stride elements between rows */
  int64_t x_stride;
  const void* weight;       /* [3 * H * D, K] (nn.Linear layout), weight_stride elements between rows */
  int64_t weight_stride;
  const void* bias;         /* optional [3 * H * D], 16-byte aligned */
  const float* cos;         /* [T, D] fp32 */
  const float* sin;         /* [T, D] fp32 */
  int64_t cs_stride_t;      /* row stride of cos and sin (a multiple of 4) */
  void* out;                /* [T, 3, H, D]: out_stride elements between token rows (>= 3 * H * D);
                               the x W^T + b of q and k rotated as HF rotates them, v as projected */
  int64_t out_stride;
  int32_t tokens;           /* T (0: nothing to do) */
  int32_t in_features;      /* K, a positive multiple of 64 */
  int32_t heads;            /* H, a multiple of 4 */
  int32_t head_dim;         /* D, 64 */
  int32_t dtype;            /* AICAS_DTYPE_F16 or AICAS_DTYPE_BF16, shared by x, weight, bias, out */
} aicas_vision_qkv_params;

AICAS_API int aicas_vision_qkv_rope(const aicas_vision_qkv_params* p, void* stream);

/* ------------------------------------------------------------------------ */
/* Decode-side weight-streaming products: Y = epilogue(X' W^T) for a few rows */
/* X (the batch of one decode step) on the tensor cores.                      */
/* ------------------------------------------------------------------------ */
#define AICAS_LINEAR_MAX_SEGMENTS 4
#define AICAS_LINEAR_MAX_ROWS 32
#define AICAS_LINEAR_STORE 0    /* out_i = X' W_i^T for every segment i */
#define AICAS_LINEAR_RESIDUAL 1 /* out = residual + round(X' W^T) (one segment; out may alias residual) */
#define AICAS_LINEAR_SWIGLU 2   /* out = silu(round(X' Wg^T)) * round(X' Wu^T): segment 0 gate, 1 up */
#define AICAS_LINEAR_NO_PDL 1   /* flags: launch without programmatic dependent launch */
#define AICAS_LINEAR_STREAM_K 2 /* flags: split K across all SMs with stream-K ranges even when the
                                   output has few tiles (default there: a CTA cluster per tile) */

typedef struct aicas_linear_segment {
  const void* weight;    /* [rows, in_features] with weight_stride elements between rows */
  int64_t weight_stride;
  void* out;             /* [batch, rows] with out_stride elements between batch rows */
  int64_t out_stride;
  int32_t rows;          /* output features of this segment */
} aicas_linear_segment;

typedef struct aicas_linear_params {
  const void* x;         /* [batch, in_features], x_stride elements between rows */
  int64_t x_stride;
  int32_t batch;         /* 1 .. AICAS_LINEAR_MAX_ROWS (0: nothing to do) */
  int32_t in_features;   /* multiple of 8 */
  const void* norm_weight; /* optional [in_features]: X' = RMSNorm(X) * norm_weight, rounded as
                              HF Qwen3VLTextRMSNorm rounds (modeling_qwen3_vl.py:398-403);
                              NULL: X' = X */
  float eps;
  int32_t mode;          /* AICAS_LINEAR_* */
  const void* residual;  /* RESIDUAL: [batch, rows] */
  int64_t residual_stride;
  int32_t num_segments;  /* 1 .. 4 (SWIGLU: 2, equal rows) */
  aicas_linear_segment seg[AICAS_LINEAR_MAX_SEGMENTS];
  int32_t dtype;         /* AICAS_DTYPE_F16 or AICAS_DTYPE_BF16, shared by every tensor */
  int32_t flags;         /* AICAS_LINEAR_NO_PDL */
  float* sumsq_out;       /* optional (one segment, STORE or RESIDUAL): [batch] fp32 receives the
                             sum of squares of each row of the (rounded) output -- the statistics
                             of the next RMSNorm, written by the last CTA to finish */
  const float* x_sumsq;   /* optional with norm_weight: [batch] fp32 sums of squares of the rows of x
                             (a previous call's sumsq_out); x is then copied by TMA and normalised in
                             shared memory instead of re-reading it for the statistics */
} aicas_linear_params;

/* Bytes of zero-initialised workspace aicas_decode_linear needs (tile counters
   and split partials); the kernel leaves the counters zeroed again. */
AICAS_API size_t aicas_linear_workspace_bytes(const aicas_linear_params* p);
AICAS_API int aicas_decode_linear(const aicas_linear_params* p, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ------------------------------------------------------------------------ */
/* Library queries.                                                           */
/* ------------------------------------------------------------------------ */
/* "aicas_b200 <version> sm_100a abi <n>" */
AICAS_API const char* aicas_version(void);

/* Bit set of AICAS_CAP_* features compiled into this library. */
#define AICAS_CAP_DECODE 1u
#define AICAS_CAP_MERGE 2u
#define AICAS_CAP_PREFILL_TCGEN05 4u
#define AICAS_CAP_VARLEN_TCGEN05 8u
#define AICAS_CAP_ROPE_APPEND 16u
#define AICAS_CAP_PEER_EXCHANGE 32u
#define AICAS_CAP_DECODE_LINEAR 64u
#define AICAS_CAP_VISION_ROPE 128u
#define AICAS_CAP_VISION_QKV 256u
AICAS_API uint32_t aicas_capabilities(void);

/* Message of the last failed call on this thread ("" if none). */
AICAS_API const char* aicas_last_error(void);

/* Reads (and optionally clears) the device-side error word of the current
   device: AICAS_DEVERR_* bits set by kernels whose bounded waits gave up.
   Synchronises the device; meant for tests and health checks, not hot loops. */
AICAS_API int aicas_device_error_flags(uint32_t* flags, int clear);

#ifdef __cplusplus
}
#endif

#endif /* AICAS_B200_H */
