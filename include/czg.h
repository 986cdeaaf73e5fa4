/*
 * czg.h -- C ABI of the B200 (sm_100a) compress-zip engine: the model forward,
 * the integer CDF and the arithmetic coder, batched over many chunks.
 *
 * It replaces the per-chunk loops of the reference CLI
 * (rust/src/main.rs:206-238 compress, rust/src/main.rs:377-396 decompress) and
 * the crate API those loops drive:
 *   Model::new / Model::forward / Model::get_cumfreqs   rust/src/model.rs:315,362,483
 *   ArithEncoder::{new, encode_symbol, finish}           rust/src/arith_coder.rs:28,80,122
 *   ArithDecoder::{new, decode_symbol}                   rust/src/arith_coder.rs:153,195
 * The tokenizer, the CZIPv1 container and the brotli/zstd outer layer stay on
 * the host.  Output is bit-identical to the reference crate.
 *
 * Conventions: plain pointers and sizes; caller-owned buffers; every entry point
 * returns an int status (CZG_OK = 0); nothing panics or aborts across the ABI.
 * One context per device.  Calls on one context are serialised by the caller
 * (the context runs its work on its own CUDA stream).  Multi-GPU use = one
 * context per device, each driven by its own host thread.
 */
#ifndef CZG_H
#define CZG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct czg_ctx czg_ctx;

enum czg_status {
    CZG_OK = 0,
    CZG_E_ARG = 1,          /* null pointer, inconsistent sizes                         */
    CZG_E_MODEL = 2,        /* .czm bytes malformed, tensor missing or of the wrong dtype */
    CZG_E_UNSUPPORTED = 3,  /* a shape the reference cannot run (it would panic)        */
    CZG_E_CAPACITY = 4,     /* output buffer too small; *out_needed holds the size      */
    CZG_E_DEVICE = 5,       /* CUDA error (message in czg_last_error)                   */
    CZG_E_TIMEOUT = 6,      /* a bounded device-side wait expired                       */
    CZG_E_TOKEN = 7,        /* token id >= vocab_size (the reference would panic)       */
    CZG_E_CHUNK = 8,        /* chunk longer than the model's context / KV cache         */
    CZG_E_LIMIT = 9         /* request beyond a fixed size limit of the entry point      */
};

/* Model facts a host driver needs (rust/src/model.rs:19-46). */
typedef struct {
    int32_t vocab_size, n_layers, n_heads, n_kv_heads, d_model, d_ff, head_dim;
    int32_t max_seq_len, context_length;
    uint32_t coef_q24, target_total;
} czg_model_info;

/* Device-side timing of the last compress/decompress call, from CUDA events on
 * the context's stream.  kernel_ms[i] is the summed duration of kernel class i
 * (names from czg_kernel_name), launches[i] its launch count. */
#define CZG_MAX_KERNEL_CLASSES 24
typedef struct {
    double total_ms;                 /* first launch to last completion, device clock */
    double h2d_ms, d2h_ms;           /* copies inside the call                        */
    uint64_t h2d_bytes, d2h_bytes;
    uint64_t n_tokens, n_chunks;
    uint32_t n_classes;
    double kernel_ms[CZG_MAX_KERNEL_CLASSES];
    uint64_t launches[CZG_MAX_KERNEL_CLASSES];
} czg_stats;

/* Load a .czm model (safetensors bytes, rust/src/model.rs:108-274 and
 * rust/src/safetensors.rs:287-376) onto `device` and make a context
 * (Model::new, rust/src/model.rs:315-351). */
int czg_ctx_create(int device, const uint8_t *czm, size_t czm_len, czg_ctx **out);
void czg_ctx_destroy(czg_ctx *ctx);

/* Message of the last failed call on ctx (or of the last failed czg_ctx_create
 * in this thread when ctx is NULL).  Valid until the next call on ctx. */
const char *czg_last_error(const czg_ctx *ctx);

int czg_model_info_get(const czg_ctx *ctx, czg_model_info *out);

/* Upper bound of the compressed bytes of n_chunks chunks holding n_tokens
 * tokens in total (at most 32 renormalisation bits per symbol plus the final
 * bit, rust/src/arith_coder.rs:101-130). */
uint64_t czg_compress_bound(uint64_t n_tokens, uint64_t n_chunks);

/* Compress chunks (the loop body of rust/src/main.rs:206-238 for every chunk).
 * tokens: host array; chunk i is tokens[chunk_starts[i] .. chunk_starts[i+1])
 * (chunk_starts has n_chunks+1 entries).  Each chunk starts from BOS 1022 at
 * position 0 with an empty KV cache.  The encoded chunks are written to `out`
 * back to back in chunk order, chunk i's length to out_lens[i].
 * out == NULL: only *out_needed = czg_compress_bound(...) is returned.
 * out_cap too small: CZG_E_CAPACITY with *out_needed = the exact total. */
int czg_compress_chunks(czg_ctx *ctx, const uint32_t *tokens, const uint64_t *chunk_starts,
                        uint32_t n_chunks, uint8_t *out, uint64_t out_cap, uint32_t *out_lens,
                        uint64_t *out_needed);

/* As czg_compress_chunks with the token ids already in device memory
 * (d_tokens on this context's device).  The encoded bytes and lengths are still
 * returned in host memory. */
int czg_compress_chunks_device(czg_ctx *ctx, const uint32_t *d_tokens,
                               const uint64_t *chunk_starts, uint32_t n_chunks, uint8_t *out,
                               uint64_t out_cap, uint32_t *out_lens, uint64_t *out_needed);

/* Decompress chunks (the loop body of rust/src/main.rs:377-396 for every chunk).
 * data: host bytes, chunk i is data[data_starts[i] .. data_starts[i+1]);
 * n_tokens[i] tokens are decoded for it (reads past its end see zero bits,
 * rust/src/arith_coder.rs:176-190).  Tokens of chunk i land at
 * out_tokens + sum(n_tokens[0..i)).  Results of 4 MB and more leave the device
 * through a page-locked staging buffer that the context keeps (grown to the
 * largest such result up to CZG_COPY_STAGING_BYTES, default 256 MB, larger ones in
 * pieces; freed by czg_ctx_destroy) and host threads copy on. */
int czg_decompress_chunks(czg_ctx *ctx, const uint8_t *data, const uint64_t *data_starts,
                          const uint32_t *n_tokens, uint32_t n_chunks, uint32_t *out_tokens);

/* Run this context's work on `stream` (a cudaStream_t of the context's device;
 * NULL restores the context's own stream).  Lets a caller order the engine's
 * kernels with its own work and time them with events on its stream.  (No
 * counterpart in the reference, which has no device streams.) */
int czg_set_stream(czg_ctx *ctx, void *stream);

/* Per-kernel timing: when on, every kernel launch is bracketed by CUDA events
 * and czg_last_stats reports time per kernel class (kernel_ms); off (the
 * default) only the whole call is timed (total_ms), which avoids the events'
 * cost (about 15% of a batched decompression with its thousands of small
 * launches).  (No counterpart in the reference.) */
int czg_set_kernel_timing(czg_ctx *ctx, int on);

/* Statistics of the last compress/decompress call on ctx. */
int czg_last_stats(const czg_ctx *ctx, czg_stats *out);
const char *czg_kernel_name(uint32_t kernel_class);

/* Per-position intermediates of one chunk computed on the GPU, for parity
 * localisation against the CPU oracle.  Any output may be NULL.
 * logits: [n][vocab] int32; lohi: [n][2] (sym_low, sym_high of the coder);
 * attn: [n][n_layers][d_model] attention outputs; final_in: [n][d_model]. */
int czg_debug_trace(czg_ctx *ctx, const uint32_t *tokens, uint32_t n, int32_t *logits,
                    uint32_t *lohi, int8_t *attn, int8_t *final_in);

/* The encoder of czg_compress_chunks run alone on given coder intervals, for
 * testing it against the reference's ArithEncoder (rust/src/arith_coder.rs:80-130)
 * on crafted interval sequences.  lohi: host array of (sym_low, sym_high) pairs,
 * chunk i taking pairs chunk_starts[i] .. chunk_starts[i+1]; each pair must
 * satisfy sym_low < sym_high <= target_total.  Output as czg_compress_chunks. */
int czg_debug_encode_intervals(czg_ctx *ctx, const uint32_t *lohi, const uint64_t *chunk_starts,
                               uint32_t n_chunks, uint8_t *out, uint64_t out_cap, uint32_t *out_lens,
                               uint64_t *out_needed);

/* Allocation-free encoder: intervals -> packed chunk bytes.  (No counterpart in
 * the reference; it is the encoder of the compress path, rust/src/arith_coder.rs
 * run per chunk, for callers that may not allocate device memory.)
 *
 * Some callers cannot call cudaMalloc/cudaFree: their device memory belongs to
 * another allocator (a framework's caching allocator or a fixed arena sized at
 * start-up) that must stay the only owner, so the library may not grow its own
 * allocations behind it.  This entry point takes every input and output in
 * device memory the caller already owns, and keeps its working storage in one
 * fixed array inside the library (12 MiB of device memory per GPU that loads
 * the library, held until the process exits).  It calls no allocating routine.
 *
 * d_lohi: device array of n_tokens (sym_low, sym_high) pairs, chunk by chunk;
 * d_chunk_len: device array of n_chunks token counts, which must sum to
 * n_tokens (checked on the device: otherwise CZG_E_ARG, and nothing is read past
 * the intervals or written);
 * target_total: the model's target total (czg_model_info.target_total).
 * Encoded chunks are packed back to back into d_out (out_cap bytes), chunk i's
 * length goes to d_out_lens[i], the packed size to *out_bytes.  Runs on
 * `stream` and waits for it before returning.
 * Limits: n_chunks <= CZG_STATIC_MAX_CHUNKS, n_tokens <= CZG_STATIC_MAX_TOKENS
 * (else CZG_E_LIMIT); a too small out_cap gives CZG_E_CAPACITY with the needed
 * size in *out_bytes.
 * The first call on a device looks up the array's device address (with that
 * device current) and keeps it for that device's context; a call after a
 * cudaDeviceReset looks it up again.  Make the first call on each device, and
 * the first after a reset, before any stream capture.  All calls
 * share the array and each call clears what must start at zero; calls whose
 * work overlaps on the GPU race on it and must be serialised by the caller. */
#define CZG_STATIC_MAX_CHUNKS 16384
#define CZG_STATIC_MAX_TOKENS 2097152
int czg_encode_intervals_static(const uint32_t *d_lohi, const uint32_t *d_chunk_len,
                                uint32_t n_chunks, uint64_t n_tokens, uint32_t target_total,
                                uint8_t *d_out, uint64_t out_cap, uint32_t *d_out_lens,
                                uint64_t *out_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif
