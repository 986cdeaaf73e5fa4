// kernels.h -- host-side launchers of the sm_100a kernels (one per file).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace czg {

// Kernels of the lockstep decode step launch with the programmatic-dependent-launch
// attribute while this is set on the calling thread (common.cuh: launch_k).
inline thread_local bool g_pdl_launch = false;

// bits of the device error word
constexpr int kErrToken = 1;     // token id >= vocab
constexpr int kErrOverflow = 2;  // an encoded chunk outgrew its slot
constexpr int kErrTimeout = 4;   // a bounded device wait gave up

// per-device one-time set-up (shared-memory opt-ins); call with the device current
void kernels_init();

// rows.cu
void launch_rows(const uint32_t *tokens, const int *chunk_row0, const int *chunk_len,
                 const uint64_t *chunk_tok0, int n_chunks, int vocab, uint32_t *tok_in,
                 uint32_t *tok_out, int *pos, int *rowchunk, int *err, cudaStream_t st);
// inv_tab: inv_rms_q15 by floor(sum_sq / d), kInvTabEntries entries, from launch_inv_table.
// x_res: the residual stream, int16 when res16 (exact for n_layers <= 128), else int32
constexpr int kInvTabEntries = 16384;
void launch_inv_table(int eps, uint16_t *tab, cudaStream_t st);
// store_res false: x_res is not written (the residual of layer 0 is then re-read from
// the embedding by the first residual norm, whose embed / tok_in are given)
void launch_embed_norm(const uint32_t *tok_in, const int8_t *embed, const int8_t *norm_w, int M,
                       int d, const uint16_t *inv_tab, void *x_res, bool res16, bool store_res, int8_t *xn,
                       cudaStream_t st);
// xn[r] = xn_tab[tok_in[r]]: the first pre-norm output from the per-token table of
// normalised embedding rows (d % 16 == 0)
void launch_xn_gather(const uint32_t *tok_in, const int8_t *xn_tab, int M, int d, int8_t *xn, cudaStream_t st);
// embed != nullptr: the residual input is embed[tok_in[r]] instead of x_res;
// store_res false: the updated residual is not written back (the model's last norm)
void launch_residual_norm(const int8_t *o, const int8_t *post_w, const int8_t *next_w, int M, int d,
                          const uint16_t *inv_tab, const uint32_t *tok_in, const int8_t *embed, bool store_res,
                          void *x_res, bool res16, int8_t *xn, cudaStream_t st);
void launch_kv_prep(const int8_t *qkv, int ldq, int d, const int *pos, const int16_t *rope_cos,
                    const int16_t *rope_sin, int M, int8_t *kv, cudaStream_t st);
// the per-chunk streaming layout (see rows.cu): chunk c from (chunk_row0[c] + 32 c) * 128
// bytes of kv, which holds (rows + 32 * chunks) * 128 bytes
void launch_kv_prep_split(const int8_t *qkv, int ldq, int d, const int *pos, const int *rowchunk,
                          const int *chunk_row0, const int *chunk_len, const int16_t *rope_cos,
                          const int16_t *rope_sin, int M, int8_t *kv, cudaStream_t st);

// GEMM epilogues (gemm_tc.cu): C[M,N] = A[M,K] . B[N,K]^T in int8 -> int32, then one of
enum GemmEpilogue {
    kEpiRequant = 0,   // out int8 [M][ldo] = requant(acc)
    kEpiReglu = 1,     // B rows interleaved (gate_j, up_j): out int8 [M][ldo], column j
    kEpiInt32 = 2,     // out int32 [M][ldo]
    kEpiRequantKv = 3  // the QKV projection: requant as kEpiRequant for the query columns
                       // [0, d); the key and value columns [d, d + 128) go, the key
                       // rotated, to the per-chunk split layout of k_kv_prep_split (KvSplit)
};

// Where kEpiRequantKv writes the keys and values: row r is position r - chunk_row0[c]
// of chunk c = rowchunk[r]; the layout is k_kv_prep_split's (rows.cu).
struct KvSplit {
    const int *rowchunk = nullptr, *chunk_row0 = nullptr, *chunk_len = nullptr;
    const int16_t *rope_cos = nullptr, *rope_sin = nullptr;
    int8_t *kv = nullptr;
    int d = 0;
};

// gemm_tc.cu: the GEMM on tcgen05 (kind::i8) with TMA-staged operands and
// TMA stores of the output.  A TcMatrix is a TMA descriptor of a row-major
// [rows][K] int8 matrix read in boxes of 128 bytes of K by box_rows rows (128 for
// A, tc_bn_for(N) for B).  Needs K % 128 == 0, N % 128 == 0 (N % 256 == 0 for
// ReGLU), a 16-byte aligned output whose row pitch is a multiple of 16 bytes.
// Returns false (nothing launched) when a shape or the output map is unsupported.
struct TcMatrix {
    alignas(64) unsigned char map[128];   // CUtensorMap
    uint64_t rows = 0, K = 0;
    int box_rows = 0;
};
int tc_bn_for(int N);   // output tile width for N (0: unsupported)
bool tc_make_matrix(TcMatrix &m, const int8_t *base, uint64_t rows, uint64_t K, int box_rows);
void gemm_tc_init();
// head_cdf.cu: the head GEMM and the coder interval in one kernel (A = final-norm
// output, B = head weight as TcMatrix; V % 256 == 0, lut4k[0] == 65535, |logit| < 2^30).
// false: unsupported shape, nothing launched.
void head_cdf_init();
bool launch_head_cdf(const TcMatrix &A, const TcMatrix &B, int M, int V, int K, const uint32_t *sym,
                     const uint16_t *lut4k, uint32_t c8, uint32_t total, uint2 *lohi, int *err, cudaStream_t st);
bool launch_gemm_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int epi, int mult, int shift,
                    void *out, int ldo, int *err, cudaStream_t st, const KvSplit *kvs = nullptr);

// the FP32 requantisation form (gemm_tc.cu, mode 3) of (mult, shift), or false
bool requant_fp32(int mult, int shift, float *mf, float *c2, int *clamp_a);
// gemm_norm.cu: O / down projection (x . W^T, FP32 requantisation) with the post norm,
// residual add and next pre-norm in the epilogue (rows.cu's k_residual_norm fused):
// B = the weight as a TcMatrix read in boxes of d/2 rows; embed != nullptr: the
// residual is embed[tok_in[r]] (written to x_res); store_res false: not written back.
// false: unsupported (d not 256/384/512, or no FP32 requantisation form), nothing launched.
void gemm_norm_init();
bool gemm_norm_supported(int d);
bool launch_gemm_norm(const TcMatrix &A, const TcMatrix &B, int M, int d, int K, int mult, int shift,
                      const int8_t *post_w, const int8_t *next_w, const uint16_t *inv_tab, const uint32_t *tok_in,
                      const int8_t *embed, bool store_res, void *x_res, bool res16, int8_t *xn, int *err,
                      cudaStream_t st);

void attention_init();
// attention_mma.cu: tensor-core version, K/V of a chunk staged in shared memory for
// chunks of at most 1024 positions (launch_attention_mma_stream for longer ones);
// lut4k = exp_q16 tabulated by t256 <= 4096 (entries from 4096 on are 1); exp0: lut4k[0] == 65535;
// score_mode: 0 exact FP32 scores (all |score_mult| < 2^19), 1 32-bit (< 2^27), 2 64-bit saturating
bool attention_mma_fits(int max_len);
void attention_mma_init();
// Tensor-core decode attention over the split KV layout: one warp per stream, the
// heads as the rows of the attention tile (n_heads <= 8); cache_ld = 128 * len,
// len % 32 == 0.
bool attention_decode_mma_ok(int n_heads);
// also appends key p and value p (columns kd..kd+127 of each qkv row) to the cache
void launch_attention_decode_mma(const int8_t *qkv, int ldq, int kd, int8_t *kvc, size_t cache_ld, int M, int p,
                                 int n_heads, const int32_t *score_mult, const int8_t *sink_key,
                                 const int16_t *rope_cos, const int16_t *rope_sin, const uint16_t *lut4k,
                                 int score_mode, bool exp0, int8_t *out, int ldo, cudaStream_t st);
void launch_attention_mma(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                          const int *chunk_len, int n_chunks, int max_len, int n_heads,
                          const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                          const int16_t *rope_sin, const uint16_t *lut4k, int score_mode, bool exp0,
                          int8_t *out, int ldo, cudaStream_t st);
// Chunks of any length: K and V in the streaming layout of launch_kv_prep_split,
// chunk i of the launch at chunk_kvoff[i] * 128 bytes of kv; chunks longest first
// (max_len = chunk 0's length); a persistent grid takes tasks from task_ctr (one
// device int, zeroed here on the stream)
void launch_attention_mma_stream(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                                 const int *chunk_len, const int *chunk_kvoff, int n_chunks, int max_len, int n_heads,
                                 const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                                 const int16_t *rope_sin, const uint16_t *lut4k, int score_mode, bool exp0,
                                 int8_t *out, int ldo, int *task_ctr, cudaStream_t st);
// attention.cu: one CTA per chunk; rows of chunk c are chunk_row0[c] ..+chunk_len[c]
void launch_attention(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                      const int *chunk_len, int n_chunks, int max_len, int n_heads,
                      const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                      const int16_t *rope_sin, const uint16_t *lut, int8_t *out, int ldo,
                      cudaStream_t st);

// decode.cu: batched decompression
struct DecState {   // arithmetic decoder state of one stream
    uint32_t low, high, code, pad;
    uint64_t bit;   // next bit of the chunk to read
};
void launch_dec_init(const uint8_t *data, const uint64_t *data_off, const uint64_t *data_len, int M,
                     DecState *st, uint32_t *tok_in, cudaStream_t stream);
// split: the tensor-core decode layout (K with permuted dims, V in 32-key tiles), see decode.cu
void launch_kv_append(const int8_t *qkv, int ldq, int d, int pos, const int16_t *rope_cos,
                      const int16_t *rope_sin, int M, int8_t *kvc, size_t cache_ld, bool split, cudaStream_t stream);
void launch_cdf_decode(const int32_t *logits, int V, int ld, const uint16_t *lut, const uint16_t *lut4k, bool exp0,
                       uint32_t coef, uint32_t total, int M, DecState *st, const uint8_t *data,
                       const uint64_t *data_off, const uint64_t *data_len, const uint64_t *tok_off, int step,
                       uint32_t *out_tok, uint32_t *tok_in, const int8_t *xn_tab, int8_t *xn, int d,
                       cudaStream_t stream);
void launch_attention_decode(const int8_t *qkv, int ldq, const int8_t *kvc, size_t cache_ld, int M, int p,
                             int n_heads, const int32_t *score_mult, const int8_t *sink_key,
                             const int16_t *rope_cos, const int16_t *rope_sin, const uint16_t *lut,
                             int8_t *out, int ldo, cudaStream_t st);

// coder.cu
// exp0: lut4k[0] == 65535 and |logit| < 2^30 (see k_cdf_lohi_reg)
void launch_cdf_lohi(const int32_t *logits, int V, int ld, const uint32_t *sym, const uint16_t *lut,
                     const uint16_t *lut4k, bool exp0, uint32_t coef, uint32_t total, int M, uint2 *lohi,
                     cudaStream_t st);
void launch_encode(const uint2 *lohi, const int *chunk_row0, const int *chunk_len, int n_chunks,
                   uint32_t total, uint8_t *slots, const uint64_t *slot_off, uint32_t *lens,
                   int *err, cudaStream_t st);
// pack_off[i] = lens[0] + ... + lens[i-1] for i <= n_chunks (on the device)
void launch_pack_offsets(const uint32_t *lens, int n_chunks, uint64_t *pack_off, cudaStream_t st);
void launch_pack(const uint8_t *slots, const uint64_t *slot_off, const uint32_t *lens,
                 const uint64_t *pack_off, int n_chunks, uint8_t *packed, cudaStream_t st);

}  // namespace czg
