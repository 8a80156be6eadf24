/*
 * laya_serve.h -- C ABI of the System One HTTP service, the `laya serve`
 * subcommand of zerodegress/laya-rust (src/main.rs:996-1204), over the
 * engines of laya_b200.h and the front end of laya_frontend.h.
 *
 * One POST endpoint takes the System One request shape and answers the
 * response JSON of laya_requests_response.  The contract of the reference is
 * kept:
 *   - status codes, checked in this order (serve_request, main.rs:1072-1138):
 *       404 {"error":"not found"}      the request target is not the endpoint
 *                                      (byte for byte: a query string is a
 *                                      different target)
 *       405 {"error":"use POST"}       any other method
 *       413 {"error":"body too large"} Content-Length above 8 MiB (MAX_BODY,
 *                                      main.rs:25), answered before the body
 *                                      is read; a chunked body is cut at 8 MiB
 *       400 {"error":"body: ..."}      the body could not be read, or is not
 *                                      UTF-8
 *       400 {"error":"invalid json: ..."}
 *       503 {"error":"server busy"}    the queue holds `queue` requests already
 *                                      (counting those still being planned)
 *       422 {"error":"..."}            parse_request / plan_items failed, or
 *                                      {"error":"no questions"}
 *                                      (Service::run, main.rs:1029-1037)
 *       500 {"error":"inference failed: ..."}  a forward failed (the
 *                                      reference answers 500 on a panic)
 *       503 {"error":"inference thread stopped"}  the service is stopping
 *       200 the response JSON
 *     with Content-Type: application/json.  Error texts of "invalid json",
 *     parse_request and plan_items are this build's JSON parser's and front
 *     end's; the codes are the contract.
 *   - the tokenizer and every engine load once, at open; an engine is
 *     created on the thread that runs it and never leaves it (the
 *     `laya-infer` thread, main.rs:1151-1160);
 *   - connection threads hand requests over a bounded queue and block for
 *     the answer; a full queue answers 503 rather than buffering.  Here they
 *     also plan their request (tokenizer, sequence layout) before queueing
 *     it, so planning runs on many threads while the GPUs work.
 * What it adds: one inference thread and engine per listed device, all
 * taking requests off the one queue (request-level data parallelism over
 * GPUs, no collective), and optionally `batch` > 1, which lets an inference
 * thread take up to `batch` queued requests at once and pack their questions
 * into shared forwards (laya_requests_pack, grouped by length across the
 * set).  batch <= 1 is the reference's run_all per request.
 *
 * Conventions are those of laya_b200.h: LAYA_OK (0) or a nonzero status with
 * the message in laya_last_error().
 */
#ifndef LAYA_SERVE_H
#define LAYA_SERVE_H

#include <stddef.h>
#include <stdint.h>

#include "laya_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct laya_server laya_server;

/* A forward supplied by the host instead of the engines: called on
 * inference thread `slot` (0 .. n_devices-1) with one batch; fills
 * logits [n*k] and act [n*2]; returns 0, or nonzero to fail the forward
 * (answered 500). */
typedef int (*laya_serve_forward_fn)(void *user, int32_t slot, const laya_req *req, float *logits, float *act);

typedef struct {
  /* GGUF model: weights, calibration (laya.temperature.*) and, unless
   * tokenizer_json is given, the embedded tokenizer.  May be NULL only with
   * a forward hook and tokenizer_json. */
  const char *model;
  const char *tokenizer_json; /* optional tokenizer.json text */
  size_t tokenizer_json_len;
  const char *addr;     /* "host:port" (IPv4); port 0 takes a free port.  NULL: "127.0.0.1:8080" */
  const char *endpoint; /* NULL: "/systemone" */
  int64_t queue;        /* queued requests before 503; <= 0: 64 */
  int32_t connections;  /* connection threads; <= 0: 4 */
  int64_t max_tokens;   /* padded-token budget per forward; <= 0: 16384 */
  const int32_t *devices; /* CUDA device of each inference thread */
  int32_t n_devices;      /* <= 0: one inference thread on device 0 */
  int32_t batch;          /* requests one inference thread takes at once; <= 1: one */
  int32_t verbose;        /* per-request status and time on stderr */
  laya_serve_forward_fn forward; /* NULL: laya_open an engine per device */
  void *forward_user;
} laya_serve_config;

/* Loads the tokenizer and opens one engine per device, each on its own
 * inference thread (Service::open, main.rs:1013-1026), then listens.  Fails
 * (and starts nothing) if a load or the bind fails. */
int laya_serve_open(const laya_serve_config *cfg, laya_server **out);
/* The bound "ip:port". */
int laya_serve_address(const laya_server *s, char *buf, size_t len);
/* Counters since open: [0] requests answered, [1] 200, [2] 400, [3] 404,
 * [4] 405, [5] 413, [6] 422, [7] 500, [8] 503, [9] forwards run, and
 * [10] the requests queued now.  Writes min(n, 11) values. */
int laya_serve_stats(const laya_server *s, int64_t *out, int n);
/* Stops taking connections; requests already queued are answered.  May be
 * called from any thread, more than once. */
int laya_serve_stop(laya_server *s);
/* Blocks until the service has stopped (after laya_serve_stop). */
int laya_serve_wait(laya_server *s);
/* Stops, waits, closes the engines (each on its own thread) and frees. */
void laya_serve_close(laya_server *s);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_SERVE_H */
