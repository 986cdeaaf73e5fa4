/* czg_tok.h -- native BPE tokenizer of a .czm model (host side, no GPU).
 *
 * Replaces the reference's CoreBPE for the shipped tokenizers
 * (rust/src/tiktoken.rs):
 *   czg_tok_create   <- load_tiktoken_json_from_bytes   (tiktoken.rs:536-563)
 *   czg_tok_encode   <- CoreBPE::encode_with_special_tokens (tiktoken.rs:498-501,
 *                       which is encode with every special token allowed, 215-268)
 *   czg_tok_encode_batch  one call over many documents on host threads
 *   czg_tok_decode   <- CoreBPE::decode_bytes            (tiktoken.rs:186-198)
 *
 * The pre-tokenizer is a hand-written scanner for one pattern, the one the
 * shipped tokenizers use (czg_tok_pattern() returns it); a JSON whose pat_str is
 * different is refused with CZG_TOK_E_PATTERN, and callers keep a general regex
 * engine for it.  Text is UTF-8; invalid UTF-8 is refused (the reference reads
 * its input with fs::read_to_string, main.rs:170).
 *
 * All functions return 0 on success or a CZG_TOK_E_* code; the message of the
 * last error on a handle is czg_tok_last_error(handle).  A handle may be used
 * from several threads at once.
 */
#ifndef CZG_TOK_H
#define CZG_TOK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    CZG_TOK_OK = 0,
    CZG_TOK_E_ARG = 1,      /* null pointer, bad size */
    CZG_TOK_E_JSON = 2,     /* the tokenizer JSON does not parse or lacks a field */
    CZG_TOK_E_PATTERN = 3,  /* pat_str is not the pattern this scanner implements */
    CZG_TOK_E_VOCAB = 4,    /* explicit_n_vocab mismatch, a byte without a token, a key outside 0..255 */
    CZG_TOK_E_UTF8 = 5,     /* input text is not valid UTF-8 */
    CZG_TOK_E_CAPACITY = 6, /* output buffer too small (the needed size is still returned) */
    CZG_TOK_E_TOKEN = 7     /* decode: unknown token id */
};

typedef struct czg_tok czg_tok;

/* The tiktoken JSON ({"pat_str", "mergeable_ranks", "special_tokens",
 * "explicit_n_vocab"}), e.g. the decompressed tokenizer.data of a .czm. */
int czg_tok_create(const char *json, size_t json_len, czg_tok **out);
void czg_tok_destroy(czg_tok *tok);
const char *czg_tok_last_error(const czg_tok *tok);
/* The pre-tokenizer pattern this scanner implements (NUL-terminated). */
const char *czg_tok_pattern(void);

/* Tokens of `text` (len bytes of UTF-8) into out[0..cap); *n_out = token count.
 * At most len tokens result, so cap = len always suffices. */
int czg_tok_encode(const czg_tok *tok, const char *text, size_t len, uint32_t *out, size_t cap, size_t *n_out);

/* n_docs documents; document i is texts[i][0..lens[i]) and its tokens go to
 * out[out_offsets[i] ..), at most lens[i] of them; n_out[i] = its count.  The
 * documents are spread over `threads` host threads (0 = all cores). */
int czg_tok_encode_batch(const czg_tok *tok, size_t n_docs, const char *const *texts, const size_t *lens,
                         uint32_t *out, const size_t *out_offsets, size_t *n_out, int threads);

/* Bytes of tokens ids[0..n) into out[0..cap); *n_out = byte count (the needed
 * size when out is NULL or too small). */
int czg_tok_decode(const czg_tok *tok, const uint32_t *ids, size_t n, uint8_t *out, size_t cap, size_t *n_out);

#ifdef __cplusplus
}
#endif
#endif
