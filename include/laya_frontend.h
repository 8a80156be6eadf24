/*
 * laya_frontend.h -- C ABI of the request front end: tokenizer, System One
 * sequence layout, packing into forwards, scoring and answers.  It turns
 * request JSON into the laya_req batches laya_forward takes (laya_b200.h)
 * and the forward outputs into the response JSON.
 *
 * Replaces, on the host side of the engine seam (zerodegress/laya-rust):
 *   src/tokenizer.rs      Tokenizer::from_json / encode (:120-265)
 *   src/systemone.rs      parse_request, render_options, build_sequence,
 *                         temperature, softmax_t, confidence, answer (:74-296)
 *   src/main.rs           plan_items (:387-410), group_by_budget (:448-468),
 *                         build_batch (:470-500), score_row (:502-518),
 *                         run_all / response (:520-557)
 * and adds what the reference does not have: planning many requests on
 * several host threads, and packing questions of different requests into one
 * forward (in dispatch order) so a GPU's forwards stay full.
 *
 * Conventions are those of laya_b200.h: every function returns LAYA_OK (0)
 * or a nonzero status, with the message in laya_last_error(); plain pointers
 * and sizes; host memory only.  A laya_tokenizer is immutable after creation
 * and may be shared by threads; a laya_requests is used by one thread at a
 * time.
 *
 * Character classes of pre-tokenisation: letters are Unicode general
 * categories L* and Nl, numbers N*, whitespace the White_Space property
 * (Rust's char::is_alphabetic also counts Other_Alphabetic combining marks as
 * letters; text with such marks can split differently).
 */
#ifndef LAYA_FRONTEND_H
#define LAYA_FRONTEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct laya_tokenizer laya_tokenizer;
typedef struct laya_requests laya_requests;

/* Tokenizer::from_json (tokenizer.rs:127-170): model.vocab, model.merges
 * (strings "a b" or pairs), added_tokens (content, id, lstrip).  Requires the
 * added tokens [CLS], [SEP], [MASK], [PAD], [UNK]. */
int laya_tokenizer_from_json(const char *json, size_t len, laya_tokenizer **out);
/* The tokenizer embedded in a model file under tokenizer.huggingface.json
 * (lib.rs:47-57). */
int laya_tokenizer_from_gguf(const char *gguf_path, laya_tokenizer **out);
/* Tokenizer::encode (tokenizer.rs:220-265) of UTF-8 text.  *n receives the
 * full token count; at most cap ids are written. */
int laya_tokenize(const laya_tokenizer *t, const char *text, size_t len, int add_special_tokens, int64_t *ids,
                  size_t cap, size_t *n);
/* The special ids: cls, sep, mask, pad, unk (5 values). */
int laya_tokenizer_specials(const laya_tokenizer *t, int64_t *ids);
void laya_tokenizer_close(laya_tokenizer *t);

/* Parses and plans n_requests request JSON documents (parse_request +
 * plan_items) on `threads` host threads (<= 0: all cores).  A request that
 * fails to parse or plan keeps its message (laya_requests_error) and
 * contributes no questions; the call itself fails only on bad arguments.
 * Questions are numbered in request order, then question order. */
int laya_requests_plan(const laya_tokenizer *t, const char *const *requests, const size_t *lens,
                       int64_t n_requests, int threads, laya_requests **out);
/* NULL when the request planned, else its error message. */
const char *laya_requests_error(const laya_requests *r, int64_t request);
int64_t laya_requests_questions(const laya_requests *r);
/* Question i: its request, sequence length, marker count and qtype. */
int laya_requests_question(const laya_requests *r, int64_t i, int64_t *request, int64_t *seq_len,
                           int64_t *n_markers, int64_t *qtype);
/* Its token ids [seq_len] and marker positions [n_markers]. */
int laya_requests_question_tokens(const laya_requests *r, int64_t i, int64_t *seq, int64_t *markers);

/* Moves the requests of parts[0..n_parts) -- planned by separate
 * laya_requests_plan calls, e.g. one per connection thread -- into one new
 * object, in that order (request j of part p follows all requests of parts
 * 0..p-1).  The parts are left with no requests and must still be closed.
 * Packing, calibration and scores of the new object start fresh. */
int laya_requests_merge(laya_requests *const *parts, int64_t n_parts, laya_requests **out);
/* Groups the questions into forwards of at most max_tokens padded tokens
 * (max_len x rows).  across_requests = 0: per request with group_by_budget
 * (questions sorted by length), the reference's run_all; 1: in dispatch
 * order across requests (a forward closes when the next question would break
 * the budget); 2: group_by_budget over all the questions of all the requests
 * (sorted by length, ties in dispatch order), the fewest forwards for a set
 * whose requests finish together.  *n_forwards receives the count. */
int laya_requests_pack(laya_requests *r, int64_t max_tokens, int across_requests, int64_t *n_forwards);
/* group_by_budget over each window of `window` consecutive requests in turn
 * (window 1: laya_requests_pack mode 0; window >= the request count: mode
 * 2).  A stream served in dispatch order keeps its order between windows
 * and gets fuller forwards inside each. */
int laya_requests_pack_windows(laya_requests *r, int64_t max_tokens, int64_t window, int64_t *n_forwards);
/* Forward f's batch shape. */
int laya_requests_forward_shape(const laya_requests *r, int64_t f, int64_t *n, int64_t *l, int64_t *k);
/* The question index of each of forward f's n rows. */
int laya_requests_forward_questions(const laya_requests *r, int64_t f, int64_t *questions);
/* build_batch (main.rs:470-500) into caller arrays: ids, att [n*l]; mpos,
 * mmask [n*k]; qtype [n] -- a laya_req's arrays. */
int laya_requests_forward_batch(const laya_requests *r, int64_t f, int64_t *ids, int64_t *att, int64_t *mpos,
                                int64_t *mmask, int64_t *qtype);
/* Calibration (systemone.rs:7-20): the three per-qtype temperatures and the
 * "qtype:size" -> temperature object of laya.temperature_by_options (JSON;
 * NULL or "{}" for none).  Default: 1, 1, 1 and none. */
int laya_requests_set_calibration(laya_requests *r, const float *temperature, const char *by_options_json);
/* score_row + answer for forward f's rows from its outputs: logits [n*k],
 * act [n*2]. */
int laya_requests_score(laya_requests *r, int64_t f, const float *logits, const float *act);
/* The response of one request (main.rs:551-557) as compact JSON:
 * {"model":"laya","answers":{...},"usage":{"input_tokens":T,"output_tokens":0}}
 * with answers in the order run_all scores the request alone (sequence
 * length, ties in question order: group_by_budget's stable sort,
 * main.rs:448-450), however its questions were packed.  *len receives the full
 * length; at most cap bytes are written (no terminator is added).  Fails if
 * a question of the request is not scored yet. */
int laya_requests_response(const laya_requests *r, int64_t request, char *buf, size_t cap, size_t *len);
void laya_requests_close(laya_requests *r);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_FRONTEND_H */
