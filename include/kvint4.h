/*
 * kvint4.h -- C ABI of libkvint4.so, the B200 (sm_100a) INT4 KV-cache library.
 *
 * Every entry point takes plain pointers, sizes and strides, returns an int
 * status (KV4_OK == 0) and never throws.  Nothing here allocates device
 * memory: outputs and any workspace are supplied by the caller.  All work is
 * enqueued on the caller's CUDA stream (passed as `void *`, a cudaStream_t;
 * NULL is the legacy default stream).
 *
 * Tensor arguments are described by kv4_tensor: a device pointer, a dtype
 * code, a 4-D shape and 4-D strides counted in ELEMENTS of that dtype (for
 * uint8 tensors elements are bytes).  Lower-rank tensors are passed with
 * leading size-1 dimensions.
 *
 * Storage format (identical to the reference, johnchmura/kv-cache-triton):
 *   packed  uint8 [..., ceil(d/G) * ceil(G/2)]  two 4-bit codes per byte,
 *           low nibble = even column, high nibble = odd column, code = q + 8
 *   scales  float [..., ceil(d/G)]  scale = max|x| / 7 over the group
 *           (1.0 for an all-zero group); value = (code - 8) * scale
 */
#ifndef KVINT4_H
#define KVINT4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
enum { KV4_F32 = 0, KV4_F16 = 1, KV4_BF16 = 2, KV4_U8 = 3 };

/* rounding of x/scale to the integer code */
enum {
  /* default: the reference's Triton GPU kernel (kernels/llama3/quantize.py:47-63):
     floor(q+0.5) / ceil(q-0.5) rounding, and both fp32 divisions (max/7 and
     x/scale) as Triton lowers fp32 `/`: PTX div.full.f32 (full-range
     approximate division), so codes and scales equal Triton's bit for bit */
  KV4_TIE_HALF_AWAY = 0,
  /* torch.round with IEEE divisions: the reference's CPU path (kernels/llama3/quantize.py:126-148) */
  KV4_TIE_HALF_EVEN = 1,
  /* half-away rounding with IEEE divisions (the Triton formula in exact
     arithmetic; what the CPU oracle restates bit for bit) */
  KV4_TIE_HALF_AWAY_IEEE = 2
};

/* status codes */
enum {
  KV4_OK = 0,
  KV4_ERR_INVALID = 1,     /* bad argument value (group_size <= 0, heads not divisible, ...) */
  KV4_ERR_DTYPE = 2,       /* unsupported dtype */
  KV4_ERR_SHAPE = 3,       /* inconsistent shapes */
  KV4_ERR_LAYOUT = 4,      /* strides/alignment the requested path cannot use */
  KV4_ERR_WORKSPACE = 5,   /* workspace missing or too small */
  KV4_ERR_CUDA = 6,        /* a CUDA runtime call failed (see kv4_last_cuda_error) */
  KV4_ERR_UNSUPPORTED = 7, /* valid request outside what the library implements */
  KV4_ERR_DEVICE = 8,      /* a kernel reported a device-side error (bounded wait expired) */
  KV4_ERR_SCRATCH_LIMIT = 9 /* kv4_attention_noalloc: request exceeds its fixed scratch area */
};

typedef struct kv4_tensor {
  void *data;
  int32_t dtype;
  int32_t pad_;
  int64_t shape[4];
  int64_t stride[4]; /* in elements */
} kv4_tensor;

/* Optional knobs for kv4_attention / kv4_attention_partial (pass NULL for defaults). */
typedef struct kv4_attn_opts {
  int32_t force_generic;   /* 1: use the generic (FFMA, any-stride) kernel */
  int32_t tiles_per_cta;   /* >0: override the split-K part length (tiles of 128 tokens per CTA) */
  int32_t max_ctas;        /* >0: cap the grid (CTAs of the one wave the split-K plan targets) */
  /* test knob: 1 = the fast path does not load each CTA's last tile and its
     bounded waits give up after 16 polls of at most 1 ms, so the wait for that
     tile expires: the kernel sets bit 1 of kv4_device_error, returns garbage
     and leaves the context usable.  0 in normal use. */
  int32_t debug_drop_last_tile;
  /* 1: launch the tensor-core kernel with programmatic stream serialization,
     so that it starts (barrier set-up, the first cache tiles in flight) while
     the kernel before it on the stream drains; it reads q, the new row, the
     workspace and writes anything only after that kernel has completed.
     Contract: the kernel launched immediately before this call on `stream`
     writes no row of this call's cache views, except row S-2 when this call
     appends row S-1 (a fused decode step on the same layer right after the
     previous one).  Ignored for the paged layout, when the call appends
     through the separate quantize kernel, and for plans of long split-K parts
     merged inside a thread-block cluster (nothing to overlap there).
     0 = ordinary stream order. */
  int32_t early_start;
} kv4_attn_opts;

/* Launch plan report (filled by kv4_attention_plan). */
typedef struct kv4_attn_plan {
  int32_t path;            /* 1 = tensor-core TMA kernel, 2 = generic kernel */
  int32_t ctas;            /* CTAs of the main kernel */
  int32_t tiles_per_cta;   /* split-K part length in 128-token tiles (fast path) */
  int32_t units;           /* (batch, kv head, column chunk) work units */
  int32_t max_parts;       /* partial slots per unit */
  int32_t kernels;         /* kernel launches one call makes */
  int64_t workspace_bytes; /* bytes the call needs in `workspace` */
} kv4_attn_plan;

/* Library version (major*10000 + minor*100 + patch) and a status message. */
int kv4_version(void);
const char *kv4_strerror(int status);
/* Last CUDA error string recorded by a call that returned KV4_ERR_CUDA. */
const char *kv4_last_cuda_error(void);

/*
 * Quantize x [n0, n1, n2, d] into packed [n0, n1, n2, >=pw] (uint8) and
 * scales [n0, n1, n2, >=ng] (f32/f16/bf16), row (i0, i1, i2) written at
 * packed/scales row (i0, i1, i2 + t_off).  x may be f32/f16/bf16 with any
 * strides.  Codes use the un-rounded fp32 scale, IEEE division x/scale, and
 * `tie_mode` rounding; the stored scale is rounded to the scales dtype.
 * Replaces kernels/llama3/quantize.py:151-186 (_quantize_int4_triton) and
 * kernels/gpt2/quantize.py:136-171.
 */
int kv4_quantize(const kv4_tensor *x, const kv4_tensor *packed, const kv4_tensor *scales,
                 int64_t t_off, int group_size, int tie_mode, void *stream);

/*
 * Quantize-on-append of both K and V in ONE launch: k, v [B, Hkv, s_new, d]
 * are quantized into the capacity buffers k_packed/v_packed [B, Hkv, cap, pw]
 * and k_scales/v_scales [B, Hkv, cap, ng] at token rows [pos, pos + s_new).
 * Replaces models/llama3/kv_cache.py:76-102 (quantize_int4 x2 + torch.cat x4)
 * and models/gpt2/kv_cache.py:42-71.
 */
int kv4_append_kv(const kv4_tensor *k, const kv4_tensor *v, const kv4_tensor *k_packed,
                  const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                  const kv4_tensor *v_scales, int64_t pos, int group_size, int tie_mode,
                  void *stream);

/*
 * out[..., :d_out] = (code - 8) * scale, d_out = out->shape[3] (<= ng*G).
 * Group slot width in nibbles is 2*packed_width/ng, as the reference's
 * view() implies.  Replaces kernels/llama3/quantize.py:237-271 and
 * kernels/gpt2/quantize.py:238-271.
 */
int kv4_dequantize(const kv4_tensor *packed, const kv4_tensor *scales, const kv4_tensor *out,
                   int group_size, void *stream);

/*
 * Fused attention over the INT4 cache, dequantizing inside the kernel:
 *   q [B, Hq, sq, d] (bf16/f16/f32), k_packed/v_packed [B, Hkv, sk, pw],
 *   k_scales/v_scales [B, Hkv, sk, ng], out [B, Hq, sq, d] (dtype of q).
 * Query head h reads KV head h / (Hq/Hkv); with is_causal, query row i sees
 * keys j <= sk - sq + i (bottom-right).  sm_scale <= 0 means d^-1/2.
 * `workspace` (device, >= kv4_attention_plan().workspace_bytes) holds
 * split-sequence partials (written from the front) and per-unit counters
 * (the LAST plan.units * 4 bytes of the `workspace_bytes` given); it may be
 * NULL when the planned size is 0.  The counter bytes must be zero before
 * the call and are zero again when it completes, so keep partial data of
 * other calls out of them (e.g. reserve a fixed zeroed tail).  Calls sharing
 * a workspace must not overlap on the GPU.
 * Replaces kernels/llama3/attention_quant.py:159-286
 * (attention_forward_quant_gqa) and kernels/gpt2/attention_quant.py:140-248
 * (attention_forward_quant, Hq == Hkv).
 */
int kv4_attention(const kv4_tensor *q, const kv4_tensor *k_packed, const kv4_tensor *k_scales,
                  const kv4_tensor *v_packed, const kv4_tensor *v_scales, const kv4_tensor *out,
                  int group_size, int is_causal, float sm_scale, void *workspace,
                  size_t workspace_bytes, const kv4_attn_opts *opts, void *stream);

/* Plan (path, grid, workspace size) of kv4_attention for the same arguments. */
int kv4_attention_plan(const kv4_tensor *q, const kv4_tensor *k_packed,
                       const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                       const kv4_tensor *v_scales, const kv4_tensor *out, int group_size,
                       int is_causal, const kv4_attn_opts *opts, kv4_attn_plan *plan);

/*
 * Decode step with the quantize-on-append fused in: k_new/v_new
 * [B, Hkv, n, d] (float, one dtype) are quantized into the LAST n rows of
 * k_packed/k_scales/v_packed/v_scales (views of sk rows that already include
 * the new positions, e.g. capacity buffers sliced to [:, :, :sk]), then q
 * attends over all sk rows; results equal kv4_append_kv(..., pos = sk - n)
 * followed by kv4_attention.  With n == 1, unit dim stride and the fast
 * path (kv4_attention_plan().path == 1) both run in ONE launch (every CTA
 * that stages the new row quantizes it itself; one CTA per (b, kv head)
 * writes it to the cache); otherwise the append kernel runs first on the
 * same stream.  Replaces the reference's per-layer decode sequence
 * QuantizedKVCache.update (models/llama3/kv_cache.py:76-102) followed by
 * attention_forward_quant_gqa (models/llama3/llama3_quant.py:59-99).
 */
int kv4_append_attention(const kv4_tensor *q, const kv4_tensor *k_new, const kv4_tensor *v_new,
                         const kv4_tensor *k_packed, const kv4_tensor *k_scales,
                         const kv4_tensor *v_packed, const kv4_tensor *v_scales,
                         const kv4_tensor *out, int group_size, int tie_mode, int is_causal,
                         float sm_scale, void *workspace, size_t workspace_bytes,
                         const kv4_attn_opts *opts, void *stream);

/*
 * Paged (block-table) INT4 cache, a layout the reference does not have (it
 * keeps one uniform-length contiguous cache per layer, models/llama3/
 * kv_cache.py:27); it serves ragged batches.  Pools:
 * k_pages/v_pages u8 [num_pages, Hkv, page, pw] and
 * k_scale_pages/v_scale_pages [num_pages, Hkv, page, ng] (page in
 * {8, 16, 32, 64, 128} tokens, rows contiguous).  Sequence b holds
 * seq_lens[b] tokens (device int32 [B]); its token t is row t % page of page
 * block_table[b * block_table_stride + t / page] (device int32).  max_seq_len
 * (host) bounds every seq_lens[b] and sizes the grid; max_blocks bounds the
 * block-table row.  q/out as for kv4_attention; is_causal aligns each
 * sequence's queries to its own last key.  Fast-path shapes only (d in
 * {64, 128, 256}, G in {32, 64, 128}), else KV4_ERR_UNSUPPORTED.  Page ids
 * outside the pool are skipped and reported by kv4_device_error (bit 2).
 */
int kv4_attention_paged(const kv4_tensor *q, const kv4_tensor *k_pages,
                        const kv4_tensor *k_scale_pages, const kv4_tensor *v_pages,
                        const kv4_tensor *v_scale_pages, const int32_t *block_table,
                        int64_t block_table_stride, int64_t max_blocks, const int32_t *seq_lens,
                        int64_t max_seq_len, const kv4_tensor *out, int group_size, int is_causal,
                        float sm_scale, void *workspace, size_t workspace_bytes,
                        const kv4_attn_opts *opts, void *stream);

/* Plan of kv4_attention_paged (grid, workspace size) for the same shapes. */
int kv4_attention_paged_plan(const kv4_tensor *q, const kv4_tensor *k_pages,
                             const kv4_tensor *k_scale_pages, const kv4_tensor *v_pages,
                             const kv4_tensor *v_scale_pages, int64_t max_blocks,
                             int64_t max_seq_len, int group_size, const kv4_attn_opts *opts,
                             kv4_attn_plan *plan);

/*
 * Quantize-on-append into a paged cache: k, v [B, Hkv, n, d] (float);
 * row (b, h, i) goes to page slot_mapping[b * n + i] / page, row
 * slot_mapping[b * n + i] % page of head h (device int32 [B * n]; negative
 * or out-of-pool slots are skipped).  Same arithmetic as kv4_append_kv.
 */
int kv4_append_kv_paged(const kv4_tensor *k, const kv4_tensor *v, const kv4_tensor *k_pages,
                        const kv4_tensor *k_scale_pages, const kv4_tensor *v_pages,
                        const kv4_tensor *v_scale_pages, const int32_t *slot_mapping,
                        int group_size, int tie_mode, void *stream);

/*
 * Sequence-shard partial of kv4_attention (new; the reference has no
 * multi-GPU layer, it relies on accelerate device_map placement,
 * benchmarks/llama3/run_llama3_benchmark.py:115-121).  The cache slice holds
 * global key positions [k_offset, k_offset + sk) of a sequence of sk_total
 * keys.  Writes part_o [B, Hq, sq, d] (f32, normalised within the shard) and
 * part_lse [B, Hq, sq, 1] (f32, natural-log sum of exp of the scaled scores;
 * -inf where the shard holds no visible key).
 */
int kv4_attention_partial(const kv4_tensor *q, const kv4_tensor *k_packed,
                          const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                          const kv4_tensor *v_scales, const kv4_tensor *part_o,
                          const kv4_tensor *part_lse, int64_t k_offset, int64_t sk_total,
                          int group_size, int is_causal, float sm_scale, void *workspace,
                          size_t workspace_bytes, const kv4_attn_opts *opts, void *stream);

/*
 * Log-sum-exp merge of n_parts shard partials: parts_o f32 contiguous
 * [n_parts, rows, d], parts_lse f32 contiguous [n_parts, rows];
 * out [B, Hq, sq, d] with B*Hq*sq == rows (any float dtype, any strides).
 * The merge step of the sequence-sharded multi-GPU decode (new layer).
 */
int kv4_lse_combine(const float *parts_o, const float *parts_lse, int64_t n_parts,
                    const kv4_tensor *out, void *stream);

/*
 * Sequence-shard exchange and merge in one launch, over peer memory (the
 * step kv4_lse_combine takes after an all-gather, with no collective
 * library and no host in the loop; capturable in a CUDA graph).  Every
 * rank owns a buffer of kv4_lse_exchange_bytes(rows, d, world) bytes,
 * zeroed before first use, reachable from every other rank's GPU
 * (symmetric memory / CUDA IPC); peer_bufs is a DEVICE array of the
 * world buffer addresses as seen from this GPU.  The kernel writes this
 * rank's partial (part_o f32 [rows, d], part_lse f32 [rows], natural-log
 * lse, as kv4_attention_partial emits them) into every buffer, each value
 * paired with the call's epoch in one 8-byte store, waits until every
 * rank's values carry the epoch (bounded: 2 s, then bit 4 of
 * kv4_device_error is set and the merge proceeds on what is there) and
 * writes the log-sum-exp merge to
 * out [B, Hq, sq, d] (B*Hq*sq == rows).  state: this rank's two zeroed
 * uint32 in device memory that count the calls (every rank makes the same
 * calls in the same order; the count picks the flag value and which of
 * two buffer halves a call uses).  No counterpart in the reference (it has
 * no multi-GPU decode).
 */
int64_t kv4_lse_exchange_bytes(int64_t rows, int d, int world);
int kv4_lse_exchange(const float *part_o, const float *part_lse, int64_t rows, int d,
                     void *const *peer_bufs, int world, int rank, uint32_t *state,
                     const kv4_tensor *out, void *stream);

/*
 * kv4_attention without a workspace argument, for callers that cannot
 * allocate device memory at the call site (no allocator reachable from
 * their runtime, or a serving step that must not touch the allocator).  It
 * has no counterpart in the reference.  Same arguments and results as
 * kv4_attention; the split-sequence partials go to a scratch area of
 * 4 MiB compiled into the library (each GPU that loads the library keeps it
 * until exit; at most 16384 work units and 4 MiB - 64 KiB of partials,
 * otherwise KV4_ERR_SCRATCH_LIMIT).  Nothing is allocated.  The first call on
 * a device looks up the area's device address (make that first call before
 * any stream capture).  All calls share the area: calls that overlap on the
 * GPU race and must be serialised by the caller.  `stream` must belong to
 * the current device (else KV4_ERR_INVALID).  The looked-up address is kept
 * for the life of the process: do not use the library across a device reset.
 */
int kv4_attention_noalloc(const kv4_tensor *q, const kv4_tensor *k_packed,
                          const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                          const kv4_tensor *v_scales, const kv4_tensor *out, int group_size,
                          int is_causal, float sm_scale, void *stream);

/*
 * Fused prefill attention on the tensor cores (tcgen05, tensor-memory
 * accumulators): the same result as kv4_attention for a query block, with
 * K/V dequantized tile by tile in shared memory (never written to HBM).
 * Supported: q/out/scales bf16, d == 128, packed rows of exactly 64 bytes
 * (token stride 64, 16-byte aligned planes and batch/head strides), scales
 * [.., d/G] contiguous per token, G in {16, 32, 64, 128}, 128 % (Hq/Hkv) == 0,
 * B * Hkv <= 65535, and for is_causal sq <= sk (bottom-right alignment:
 * query i sees keys j <= sk - sq + i).  Anything else returns
 * KV4_ERR_UNSUPPORTED / KV4_ERR_LAYOUT and the caller uses kv4_attention.
 * sm_scale <= 0 means 1/sqrt(d).  No workspace.  The tensor-core operands
 * are f16: dequantized K/V values are exact in f16 while |value| < 65504;
 * a scale above 65504/8 sets bit 8 of kv4_device_error (output not valid).
 * Replaces the prefill branch (sq > 1) of kernels/llama3/attention_quant.py:24-152
 * (_attn_fwd_quant_gqa_kernel with IS_CAUSAL) for the shapes above.
 */
int kv4_prefill_attention(const kv4_tensor *q, const kv4_tensor *k_packed,
                          const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                          const kv4_tensor *v_scales, const kv4_tensor *out, int group_size,
                          int is_causal, float sm_scale, void *stream);

/* Read-and-clear the device error word (synchronizes the stream): bit 1 a
   bounded mbarrier wait expired, bit 2 a page id outside the pool, bit 4 a
   peer exchange wait expired, bit 8 kv4_prefill_attention met K/V values
   outside the f16 range. */
int kv4_device_error(void *stream, int *flag_out);

#ifdef __cplusplus
}
#endif
#endif /* KVINT4_H */
