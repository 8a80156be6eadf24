// The System One HTTP service (include/laya_serve.h): `laya serve` of
// laya-rust src/main.rs:996-1204 over this library's engines and front end.
//
// Threads
//   - `connections` connection threads: each accepts a connection and serves
//     its requests in turn (HTTP/1.1 keep-alive), checking them in the order
//     of serve_request (main.rs:1072-1138); a request that passes takes a
//     queue slot, is planned on this thread (parse_request + plan_items of
//     Service::run, main.rs:1029-1034: 422 on failure) and queued, and the
//     thread blocks on its answer.  Planning here, on many threads, keeps it
//     off the inference threads' path to the GPU;
//   - one inference thread per device: it opens its engine itself (the
//     engine never leaves that thread, main.rs:1151-1160), then takes jobs
//     off the shared bounded queue (up to `batch`, merged into one set),
//     packs them, runs their forwards, scores them and answers
//     (run_all + response, main.rs:520-557).
// The queue holds at most `queue` jobs that no inference thread has taken,
// counting those still being planned (sync_channel(queue), main.rs:1148); a
// request that finds it full is answered 503 at once.
#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/laya_frontend.h"
#include "../../include/laya_serve.h"
#include "gguf_reader.h"
#include "json.h"

namespace laya {
void set_last_error(const char* msg);  // engine.cpp: the thread's laya_last_error()

namespace serve {

constexpr size_t kMaxBody = size_t(8) << 20;  // MAX_BODY (main.rs:25)
constexpr size_t kMaxHead = size_t(64) << 10;  // request line + headers
constexpr int kSliceMs = 100;                   // poll slice: how fast stop is seen
constexpr int kIdleMs = 5000;                   // keep-alive connection idle limit
constexpr int kReadMs = 30000;                  // limit for the rest of a started request

enum Stat { kAnswered, k200, k400, k404, k405, k413, k422, k500, k503, kForwards, kNumStats };

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

std::string error_body(const std::string& msg) {
  std::string out = "{\"error\":";
  json::dump_string(msg, out);
  out += '}';
  return out;
}

// One request handed from a connection thread to an inference thread.
struct Job {
  laya_requests* plan = nullptr;  // one planned request; the inference thread closes it
  int status = 0;
  std::string out;
  bool done = false;
  std::mutex m;
  std::condition_variable cv;

  void finish(int st, std::string o) {
    std::lock_guard<std::mutex> g(m);
    status = st;
    out = std::move(o);
    done = true;
    cv.notify_all();
  }
  // finish() unless answered already
  void finish_open(int st, const std::string& o) {
    std::lock_guard<std::mutex> g(m);
    if (done) return;
    status = st;
    out = o;
    done = true;
    cv.notify_all();
  }
  void wait() {
    std::unique_lock<std::mutex> g(m);
    cv.wait(g, [&] { return done; });
  }
  ~Job() {
    if (plan) laya_requests_close(plan);
  }
};

// Strict UTF-8 (what Rust's read_to_string accepts): no overlong forms, no
// surrogates, nothing above U+10FFFF.
bool valid_utf8(const std::string& s) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  size_t i = 0, n = s.size();
  while (i < n) {
    const unsigned c = p[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    size_t len;
    unsigned lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
    } else if (c >= 0xE0 && c <= 0xEF) {
      len = 3;
      if (c == 0xE0) lo = 0xA0;
      if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      len = 4;
      if (c == 0xF0) lo = 0x90;
      if (c == 0xF4) hi = 0x8F;
    } else {
      return false;
    }
    if (i + len > n) return false;
    if (p[i + 1] < lo || p[i + 1] > hi) return false;
    for (size_t j = 2; j < len; ++j)
      if ((p[i + j] & 0xC0) != 0x80) return false;
    i += len;
  }
  return true;
}

const char* reason(int code) {
  switch (code) {
    case 100: return "Continue";
    case 200: return "OK";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 413: return "Payload Too Large";
    case 422: return "Unprocessable Entity";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
    default: return "Unknown";
  }
}

std::string lower(std::string s) {
  for (char& c : s)
    if (c >= 'A' && c <= 'Z') c = static_cast<char>(c - 'A' + 'a');
  return s;
}

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (s[a] == ' ' || s[a] == '\t')) ++a;
  while (b > a && (s[b - 1] == ' ' || s[b - 1] == '\t')) --b;
  return s.substr(a, b - a);
}

struct Server;

// A connection's buffered reader.  Every wait polls in kSliceMs slices so a
// stop is seen; a read gives up at its limit, on EOF and on stop.
struct Conn {
  int fd;
  const std::atomic<bool>* stopping;
  std::string buf;
  size_t pos = 0;

  // Reads more bytes; false on EOF, error, timeout or stop.
  bool fill(int limit_ms) {
    int waited = 0;
    for (;;) {
      if (stopping->load()) return false;
      pollfd p{fd, POLLIN, 0};
      const int r = poll(&p, 1, kSliceMs);
      if (r < 0) {
        if (errno == EINTR) continue;
        return false;
      }
      if (r == 0) {
        waited += kSliceMs;
        if (waited >= limit_ms) return false;
        continue;
      }
      char tmp[65536];
      const ssize_t got = recv(fd, tmp, sizeof tmp, 0);
      if (got < 0 && errno == EINTR) continue;
      if (got <= 0) return false;
      if (pos > 0 && pos == buf.size()) {
        buf.clear();
        pos = 0;
      }
      buf.append(tmp, static_cast<size_t>(got));
      return true;
    }
  }
  size_t avail() const { return buf.size() - pos; }
  // n bytes into out (appended); false if the stream ends first.
  bool read_exact(size_t n, std::string& out, int limit_ms) {
    while (avail() < n) {
      const size_t have = avail();
      out.append(buf, pos, have);
      pos += have;
      n -= have;
      if (!fill(limit_ms)) return false;
    }
    out.append(buf, pos, n);
    pos += n;
    return true;
  }
  // One CRLF-terminated line (CRLF removed), at most `cap` bytes.
  bool read_line(std::string& line, size_t cap, int limit_ms) {
    for (;;) {
      const size_t e = buf.find("\r\n", pos);
      if (e != std::string::npos) {
        line.assign(buf, pos, e - pos);
        pos = e + 2;
        return true;
      }
      if (avail() > cap) return false;
      if (!fill(limit_ms)) return false;
    }
  }
  bool send_all(const std::string& s) {
    size_t off = 0;
    while (off < s.size()) {
      const ssize_t w = send(fd, s.data() + off, s.size() - off, MSG_NOSIGNAL);
      if (w < 0 && errno == EINTR) continue;
      if (w <= 0) return false;
      off += static_cast<size_t>(w);
    }
    return true;
  }
};

struct Server {
  // configuration
  std::string model, tokenizer_json, addr, endpoint;
  int64_t queue_cap = 64, max_tokens = 16384;
  int connections = 4, batch = 1;
  bool verbose = false;
  std::vector<int> devices;
  laya_serve_forward_fn hook = nullptr;
  void* hook_user = nullptr;
  float temperature[3] = {1.f, 1.f, 1.f};
  std::string by_options = "{}";

  laya_tokenizer* tok = nullptr;
  int listen_fd = -1;
  std::string bound;
  std::atomic<bool> stopping{false};
  std::atomic<int64_t> stats[kNumStats];

  std::mutex qm;
  std::condition_variable qcv;
  std::deque<std::shared_ptr<Job>> q;
  int64_t reserved = 0;  // slots held by requests their connection thread is planning
  bool q_closed = false;

  std::mutex rm;
  std::condition_variable rcv;
  int reported = 0;
  std::string load_error;

  std::vector<std::thread> infer, conns;
  std::mutex jm;
  bool joined = false;

  Server() {
    for (auto& s : stats) s.store(0);
  }

  void count(int code) {
    stats[kAnswered]++;
    switch (code) {
      case 200: stats[k200]++; break;
      case 400: stats[k400]++; break;
      case 404: stats[k404]++; break;
      case 405: stats[k405]++; break;
      case 413: stats[k413]++; break;
      case 422: stats[k422]++; break;
      case 500: stats[k500]++; break;
      case 503: stats[k503]++; break;
      default: break;
    }
  }

  // ---- inference threads -------------------------------------------------
  void report(const std::string& err) {
    std::lock_guard<std::mutex> g(rm);
    if (!err.empty() && load_error.empty()) load_error = err;
    ++reported;
    rcv.notify_all();
  }

  // Takes up to `batch` jobs; blocks for the first.  Empty: closed and drained.
  std::vector<std::shared_ptr<Job>> take() {
    std::unique_lock<std::mutex> g(qm);
    qcv.wait(g, [&] { return !q.empty() || q_closed; });
    std::vector<std::shared_ptr<Job>> jobs;
    while (!q.empty() && static_cast<int>(jobs.size()) < batch) {
      jobs.push_back(std::move(q.front()));
      q.pop_front();
    }
    return jobs;
  }

  void inference_thread(int slot) {
    laya_engine* eng = nullptr;
    if (!hook) {
      if (laya_open(devices[slot], model.c_str(), &eng) != LAYA_OK) {
        report("device " + std::to_string(devices[slot]) + ": " + laya_last_error());
        return;
      }
    }
    report("");
    for (;;) {
      std::vector<std::shared_ptr<Job>> jobs = take();
      if (jobs.empty()) break;
      // nothing may escape the thread, and every job taken gets an answer
      std::string err;
      try {
        run(slot, eng, jobs);
      } catch (const std::bad_alloc&) {
        err = "out of host memory";
      } catch (const std::exception& e) {
        err = e.what();
      }
      if (!err.empty())
        for (auto& j : jobs) j->finish_open(500, error_body("inference failed: " + err));
    }
    if (eng) laya_close(eng);
  }

  // Service::run (main.rs:1029-1037) for one or more jobs.
  void run(int slot, laya_engine* eng, std::vector<std::shared_ptr<Job>>& jobs) {
    const int64_t n = static_cast<int64_t>(jobs.size());
    std::vector<bool> open(n, true);
    auto fail_open = [&](int code, const std::string& msg) {
      for (int64_t j = 0; j < n; ++j)
        if (open[j]) {
          open[j] = false;
          jobs[j]->finish(code, error_body(msg));
        }
    };
    // the connection threads planned each request; one object for the set
    laya_requests* r = nullptr;
    if (n == 1) {
      r = jobs[0]->plan;
      jobs[0]->plan = nullptr;
    } else {
      std::vector<laya_requests*> parts(n);
      for (int64_t j = 0; j < n; ++j) parts[j] = jobs[j]->plan;
      const int st = laya_requests_merge(parts.data(), n, &r);
      for (int64_t j = 0; j < n; ++j) {
        laya_requests_close(jobs[j]->plan);
        jobs[j]->plan = nullptr;
      }
      if (st != LAYA_OK) {
        fail_open(500, std::string("inference failed: ") + laya_last_error());
        return;
      }
    }
    if (laya_requests_set_calibration(r, temperature, by_options.c_str()) != LAYA_OK) {
      fail_open(500, std::string("inference failed: ") + laya_last_error());
      laya_requests_close(r);
      return;
    }
    int64_t nf = 0;
    // one request: run_all's grouping; a set taken together finishes
    // together, so it is grouped by length as a whole (fewest forwards)
    if (laya_requests_pack(r, max_tokens, n > 1 ? 2 : 0, &nf) != LAYA_OK) {
      fail_open(500, std::string("inference failed: ") + laya_last_error());
      laya_requests_close(r);
      return;
    }
    std::vector<int64_t> ids, att, mpos, mmask, qtype;
    std::vector<float> logits, act;
    for (int64_t f = 0; f < nf; ++f) {
      int64_t bn = 0, bl = 0, bk = 0;
      std::string err;
      if (laya_requests_forward_shape(r, f, &bn, &bl, &bk) != LAYA_OK) {
        err = laya_last_error();
      } else {
        const size_t nl = static_cast<size_t>(std::max<int64_t>(1, bn * bl));
        const size_t nk = static_cast<size_t>(std::max<int64_t>(1, bn * bk));
        ids.assign(nl, 0);
        att.assign(nl, 0);
        mpos.assign(nk, 0);
        mmask.assign(nk, 0);
        qtype.assign(static_cast<size_t>(std::max<int64_t>(1, bn)), 0);
        logits.assign(nk, 0.f);
        act.assign(static_cast<size_t>(std::max<int64_t>(1, bn * 2)), 0.f);
        if (laya_requests_forward_batch(r, f, ids.data(), att.data(), mpos.data(), mmask.data(), qtype.data()) !=
            LAYA_OK) {
          err = laya_last_error();
        } else {
          const laya_req req{bn, bl, bk, ids.data(), att.data(), mpos.data(), mmask.data(), qtype.data()};
          if (hook) {
            const int rc = hook(hook_user, slot, &req, logits.data(), act.data());
            if (rc != 0) err = "forward hook returned " + std::to_string(rc);
          } else if (laya_forward(eng, &req, logits.data(), act.data()) != LAYA_OK) {
            err = laya_last_error();
          }
          stats[kForwards]++;
          if (err.empty() && laya_requests_score(r, f, logits.data(), act.data()) != LAYA_OK)
            err = laya_last_error();
        }
      }
      if (!err.empty()) {
        fail_open(500, "inference failed: " + err);
        laya_requests_close(r);
        return;
      }
    }
    std::string out(4096, '\0');
    for (int64_t j = 0; j < n; ++j) {
      if (!open[j]) continue;
      size_t len = 0;
      int st = laya_requests_response(r, j, &out[0], out.size(), &len);
      if (st == LAYA_OK && len > out.size()) {
        out.resize(len);
        st = laya_requests_response(r, j, &out[0], out.size(), &len);
      }
      open[j] = false;
      if (st != LAYA_OK)
        jobs[j]->finish(500, error_body(std::string("inference failed: ") + laya_last_error()));
      else
        jobs[j]->finish(200, out.substr(0, len));
    }
    laya_requests_close(r);
  }

  // ---- connection threads ------------------------------------------------
  void respond(Conn& c, int code, const std::string& body, bool keep) {
    std::string head = "HTTP/1.1 " + std::to_string(code) + " " + reason(code) +
                       "\r\nContent-Type: application/json\r\nContent-Length: " + std::to_string(body.size()) +
                       (keep ? "\r\nConnection: keep-alive\r\n\r\n" : "\r\nConnection: close\r\n\r\n");
    head += body;
    c.send_all(head);
    count(code);
  }

  // A chunked body (RFC 9112 7.1), cut at kMaxBody (the reference reads
  // through take(MAX_BODY)); *cut tells the caller the rest is unread.
  bool read_chunked(Conn& c, std::string& body, bool* cut, std::string* why) {
    std::string line;
    for (;;) {
      if (!c.read_line(line, 4096, kReadMs)) {
        *why = "unexpected end of chunked body";
        return false;
      }
      const size_t semi = line.find(';');
      const std::string hex = trim(semi == std::string::npos ? line : line.substr(0, semi));
      if (hex.empty() || hex.size() > 15 || hex.find_first_not_of("0123456789abcdefABCDEF") != std::string::npos) {
        *why = "invalid chunk size";
        return false;
      }
      const size_t size = std::stoull(hex, nullptr, 16);
      if (size == 0) {
        do {  // trailer fields, then the empty line
          if (!c.read_line(line, 4096, kReadMs)) {
            *why = "unexpected end of chunked body";
            return false;
          }
        } while (!line.empty());
        return true;
      }
      if (body.size() + size > kMaxBody) {
        const size_t keep = kMaxBody - body.size();
        if (!c.read_exact(keep, body, kReadMs)) {
          *why = "unexpected end of chunked body";
          return false;
        }
        *cut = true;
        return true;
      }
      std::string crlf;
      if (!c.read_exact(size, body, kReadMs) || !c.read_exact(2, crlf, kReadMs) || crlf != "\r\n") {
        *why = "unexpected end of chunked body";
        return false;
      }
    }
  }

  // Serves one connection's requests; returns when it closes.
  void serve_connection(int fd) {
    Conn c{fd, &stopping};
    for (;;) {
      c.buf.erase(0, c.pos);
      c.pos = 0;
      // request line and headers
      size_t end;
      bool started = c.avail() > 0;
      while ((end = c.buf.find("\r\n\r\n", c.pos)) == std::string::npos) {
        if (c.avail() > kMaxHead) {
          respond(c, 400, error_body("request head too large"), false);
          return;
        }
        if (!c.fill(started ? kReadMs : kIdleMs)) return;
        started = true;
      }
      if (end - c.pos > kMaxHead) {  // the whole head may have come in one read
        respond(c, 400, error_body("request head too large"), false);
        return;
      }
      const auto t0 = std::chrono::steady_clock::now();
      const std::string head = c.buf.substr(c.pos, end - c.pos);
      c.pos = end + 4;
      std::vector<std::string> lines;
      for (size_t a = 0;;) {
        const size_t b = head.find("\r\n", a);
        lines.push_back(head.substr(a, b == std::string::npos ? std::string::npos : b - a));
        if (b == std::string::npos) break;
        a = b + 2;
      }
      std::string method, target, version;
      {
        const std::string& rl = lines[0];
        const size_t s1 = rl.find(' ');
        const size_t s2 = s1 == std::string::npos ? s1 : rl.find(' ', s1 + 1);
        if (s2 == std::string::npos || rl.find(' ', s2 + 1) != std::string::npos) {
          respond(c, 400, error_body("malformed request line"), false);
          return;
        }
        method = rl.substr(0, s1);
        target = rl.substr(s1 + 1, s2 - s1 - 1);
        version = rl.substr(s2 + 1);
      }
      if (version != "HTTP/1.1" && version != "HTTP/1.0") {
        respond(c, 400, error_body("unsupported HTTP version"), false);
        return;
      }
      bool chunked = false, expect100 = false, have_len = false;
      std::string conn_hdr;
      size_t clen = 0;
      for (size_t i = 1; i < lines.size(); ++i) {
        const size_t colon = lines[i].find(':');
        if (colon == std::string::npos || colon == 0) {
          respond(c, 400, error_body("malformed header"), false);
          return;
        }
        const std::string name = lower(lines[i].substr(0, colon));
        const std::string value = trim(lines[i].substr(colon + 1));
        if (name == "content-length") {
          if (value.empty() || value.size() > 18 || value.find_first_not_of("0123456789") != std::string::npos ||
              (have_len && std::stoull(value) != clen)) {
            respond(c, 400, error_body("invalid Content-Length"), false);
            return;
          }
          clen = std::stoull(value);
          have_len = true;
        } else if (name == "transfer-encoding") {
          chunked = lower(value).find("chunked") != std::string::npos;
        } else if (name == "connection") {
          conn_hdr = lower(value);
        } else if (name == "expect") {
          expect100 = lower(value) == "100-continue";
        }
      }
      bool keep = version == "HTTP/1.1" ? conn_hdr.find("close") == std::string::npos
                                        : conn_hdr.find("keep-alive") != std::string::npos;
      const bool has_body = chunked || clen > 0;
      auto log = [&](int code, const std::string& what) {
        if (!verbose) return;
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (code == 200)
          fprintf(stderr, "200 in %.2fms\n", ms);
        else
          fprintf(stderr, "%d in %.2fms: %s\n", code, ms, what.c_str());
      };
      // serve_request (main.rs:1072-1138): route, method, size, body, JSON, queue
      if (target != endpoint) {
        respond(c, 404, error_body("not found"), keep && !has_body);
        if (keep && !has_body) continue;
        return;
      }
      if (method != "POST") {
        respond(c, 405, error_body("use POST"), keep && !has_body);
        if (keep && !has_body) continue;
        return;
      }
      if (!chunked && clen > kMaxBody) {
        respond(c, 413, error_body("body too large"), false);
        return;
      }
      if (expect100 && !c.send_all("HTTP/1.1 100 Continue\r\n\r\n")) return;
      std::string body, why;
      bool cut = false;
      const bool ok = chunked ? read_chunked(c, body, &cut, &why) : c.read_exact(clen, body, kReadMs);
      if (!ok) {
        if (why.empty()) why = "unexpected end of body";
        respond(c, 400, error_body("body: " + why), false);
        log(400, "body: " + why);
        return;
      }
      if (cut) keep = false;
      if (!valid_utf8(body)) {
        const std::string m = "body: stream did not contain valid UTF-8";
        respond(c, 400, error_body(m), keep);
        log(400, m);
        if (keep) continue;
        return;
      }
      try {
        (void)json::parse(body.data(), body.size());
      } catch (const std::exception& e) {
        const std::string m = std::string("invalid json: ") + e.what();
        respond(c, 400, error_body(m), keep);
        log(400, m);
        if (keep) continue;
        return;
      }
      // a queue slot first (a full queue answers 503 before the request is
      // looked at, as in the reference), then parse_request + plan_items on
      // this thread, so the inference threads only pack and run forwards
      int busy = 0;
      {
        std::lock_guard<std::mutex> g(qm);
        if (q_closed)
          busy = 1;
        else if (static_cast<int64_t>(q.size()) + reserved >= queue_cap)
          busy = 2;
        else
          ++reserved;
      }
      if (busy) {
        const std::string m = busy == 1 ? "inference thread stopped" : "server busy";
        respond(c, 503, error_body(m), keep);
        log(503, m);
        if (keep) continue;
        return;
      }
      auto job = std::make_shared<Job>();
      int code = 0;
      std::string why2;
      {
        const char* text = body.data();
        const size_t len = body.size();
        if (laya_requests_plan(tok, &text, &len, 1, 1, &job->plan) != LAYA_OK) {
          code = 500;
          why2 = std::string("inference failed: ") + laya_last_error();
        } else if (const char* e = laya_requests_error(job->plan, 0)) {
          code = 422;  // parse_request / plan_items (Service::run, main.rs:1030-1034)
          why2 = e;
        } else if (laya_requests_questions(job->plan) == 0) {
          code = 422;
          why2 = "no questions";
        }
      }
      {
        std::lock_guard<std::mutex> g(qm);
        --reserved;
        if (!code) {
          if (q_closed) {
            code = 503;
            why2 = "inference thread stopped";
          } else {
            q.push_back(job);
          }
        }
      }
      if (code) {
        respond(c, code, error_body(why2), keep);
        log(code, why2);
        if (keep) continue;
        return;
      }
      qcv.notify_one();
      job->wait();
      respond(c, job->status, job->out, keep);
      log(job->status, job->out);
      if (!keep) return;
    }
  }

  void connection_thread() {
    while (!stopping.load()) {
      pollfd p{listen_fd, POLLIN, 0};
      const int r = poll(&p, 1, kSliceMs);
      if (r <= 0 || stopping.load()) continue;
      const int fd = accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
      if (fd < 0) continue;  // another thread took it (EAGAIN), or the peer went away
      const int one = 1;
      setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
      const timeval send_limit{kReadMs / 1000, 0};
      setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &send_limit, sizeof send_limit);
      try {
        serve_connection(fd);
      } catch (const std::exception& e) {
        // out of memory or the like: drop this connection, keep serving
        if (verbose) fprintf(stderr, "connection dropped: %s\n", e.what());
      }
      close(fd);
    }
  }

  // ---- life cycle --------------------------------------------------------
  void bind_listen() {
    const size_t colon = addr.rfind(':');
    if (colon == std::string::npos) throw Error(LAYA_E_INVALID, addr + ": want host:port");
    std::string host = addr.substr(0, colon);
    const std::string port = addr.substr(colon + 1);
    if (host.empty()) host = "0.0.0.0";
    addrinfo hints{};
    hints.ai_family = AF_INET;
    hints.ai_socktype = SOCK_STREAM;
    hints.ai_flags = AI_PASSIVE;
    addrinfo* res = nullptr;
    const int gai = getaddrinfo(host.c_str(), port.c_str(), &hints, &res);
    if (gai != 0) throw Error(LAYA_E_INVALID, addr + ": " + gai_strerror(gai));
    const int fd = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC | SOCK_NONBLOCK, 0);
    if (fd < 0) {
      freeaddrinfo(res);
      throw Error(LAYA_E_INVALID, addr + ": socket: " + strerror(errno));
    }
    const int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
    if (bind(fd, res->ai_addr, res->ai_addrlen) != 0 || listen(fd, 128) != 0) {
      const std::string e = strerror(errno);
      freeaddrinfo(res);
      close(fd);
      throw Error(LAYA_E_INVALID, addr + ": " + e);
    }
    freeaddrinfo(res);
    sockaddr_in sa{};
    socklen_t sl = sizeof sa;
    getsockname(fd, reinterpret_cast<sockaddr*>(&sa), &sl);
    char ip[INET_ADDRSTRLEN] = {0};
    inet_ntop(AF_INET, &sa.sin_addr, ip, sizeof ip);
    bound = std::string(ip) + ":" + std::to_string(ntohs(sa.sin_port));
    listen_fd = fd;
  }

  void close_queue() {
    {
      std::lock_guard<std::mutex> g(qm);
      q_closed = true;
    }
    qcv.notify_all();
  }

  // Connection threads first (no new jobs), then the inference threads,
  // which answer what is queued before they exit.
  void join_all() {
    std::lock_guard<std::mutex> g(jm);
    if (joined) return;
    for (auto& t : conns) t.join();
    close_queue();
    for (auto& t : infer) t.join();
    joined = true;
  }

  ~Server() {
    if (!joined) {  // open() failed part-way: stop what was started
      stopping.store(true);
      for (auto& t : conns)
        if (t.joinable()) t.join();
      close_queue();
      for (auto& t : infer)
        if (t.joinable()) t.join();
    }
    if (listen_fd >= 0) close(listen_fd);
    if (tok) laya_tokenizer_close(tok);
  }
};

void read_calibration(Server& s) {
  // ModelMeta::calibration (weights.rs:131): laya.temperature.{0,1,2} and
  // laya.temperature_by_options; absent keys keep the defaults
  GgufFile g(s.model);
  for (int i = 0; i < 3; ++i) {
    const GgufValue* v = g.get("laya.temperature." + std::to_string(i));
    if (v && v->has_f) s.temperature[i] = static_cast<float>(v->f);
  }
  const GgufValue* v = g.get("laya.temperature_by_options");
  if (v && v->has_s && !v->s.empty()) s.by_options = v->s;
}

template <class F>
int guard(F&& f) {
  try {
    f();
    set_last_error("");
    return LAYA_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("out of host memory");
    return LAYA_E_INVALID;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return LAYA_E_LOAD;
  }
}

}  // namespace serve
}  // namespace laya

struct laya_server {
  std::unique_ptr<laya::serve::Server> s;
};

using laya::serve::Error;

extern "C" {

int laya_serve_open(const laya_serve_config* cfg, laya_server** out) {
  return laya::serve::guard([&] {
    if (!cfg || !out) throw Error(LAYA_E_INVALID, "null argument");
    *out = nullptr;
    auto s = std::make_unique<laya::serve::Server>();
    if (cfg->model) s->model = cfg->model;
    if (cfg->tokenizer_json) s->tokenizer_json.assign(cfg->tokenizer_json, cfg->tokenizer_json_len);
    s->addr = cfg->addr ? cfg->addr : "127.0.0.1:8080";
    s->endpoint = cfg->endpoint ? cfg->endpoint : "/systemone";
    s->queue_cap = cfg->queue > 0 ? cfg->queue : 64;
    s->connections = cfg->connections > 0 ? cfg->connections : 4;
    s->max_tokens = cfg->max_tokens > 0 ? cfg->max_tokens : 16384;
    s->batch = cfg->batch > 1 ? cfg->batch : 1;
    s->verbose = cfg->verbose != 0;
    s->hook = cfg->forward;
    s->hook_user = cfg->forward_user;
    if (cfg->n_devices > 0) {
      if (!cfg->devices) throw Error(LAYA_E_INVALID, "null device list");
      s->devices.assign(cfg->devices, cfg->devices + cfg->n_devices);
    } else {
      s->devices = {0};
    }
    if (s->model.empty() && (!s->hook || s->tokenizer_json.empty()))
      throw Error(LAYA_E_INVALID, "a model path is needed (or a forward hook and tokenizer_json)");
    // Service::open (main.rs:1013-1026): tokenizer once, engines on their threads
    laya_tokenizer* tok = nullptr;
    const int st = s->tokenizer_json.empty()
                       ? laya_tokenizer_from_gguf(s->model.c_str(), &tok)
                       : laya_tokenizer_from_json(s->tokenizer_json.data(), s->tokenizer_json.size(), &tok);
    if (st != LAYA_OK) throw Error(st, laya_last_error());
    s->tok = tok;
    if (!s->model.empty()) laya::serve::read_calibration(*s);
    laya::serve::Server* sp = s.get();
    const int n = static_cast<int>(s->devices.size());
    for (int i = 0; i < n; ++i) s->infer.emplace_back([sp, i] { sp->inference_thread(i); });
    std::string load_error;
    {
      std::unique_lock<std::mutex> g(s->rm);
      s->rcv.wait(g, [&] { return s->reported == n; });
      load_error = s->load_error;
    }
    if (load_error.empty()) {
      try {
        s->bind_listen();
      } catch (const std::exception& e) {
        load_error = e.what();
      }
    }
    if (!load_error.empty()) {
      s->close_queue();
      for (auto& t : s->infer) t.join();
      s->infer.clear();
      s->joined = true;
      throw Error(LAYA_E_LOAD, load_error);
    }
    for (int i = 0; i < s->connections; ++i) s->conns.emplace_back([sp] { sp->connection_thread(); });
    *out = new laya_server{std::move(s)};
  });
}

int laya_serve_address(const laya_server* s, char* buf, size_t len) {
  return laya::serve::guard([&] {
    if (!s || !buf || len == 0) throw Error(LAYA_E_INVALID, "null argument");
    const std::string& a = s->s->bound;
    if (a.size() + 1 > len) throw Error(LAYA_E_INVALID, "buffer too small");
    memcpy(buf, a.c_str(), a.size() + 1);
  });
}

int laya_serve_stats(const laya_server* s, int64_t* out, int n) {
  return laya::serve::guard([&] {
    if (!s || !out || n < 0) throw Error(LAYA_E_INVALID, "null argument");
    for (int i = 0; i < n && i < laya::serve::kNumStats; ++i) out[i] = s->s->stats[i].load();
    if (n > laya::serve::kNumStats) {
      std::lock_guard<std::mutex> g(s->s->qm);
      out[laya::serve::kNumStats] = static_cast<int64_t>(s->s->q.size());
    }
  });
}

int laya_serve_stop(laya_server* s) {
  return laya::serve::guard([&] {
    if (!s) throw Error(LAYA_E_INVALID, "null server");
    s->s->stopping.store(true);
  });
}

int laya_serve_wait(laya_server* s) {
  return laya::serve::guard([&] {
    if (!s) throw Error(LAYA_E_INVALID, "null server");
    s->s->join_all();
  });
}

void laya_serve_close(laya_server* s) {
  if (!s) return;
  s->s->stopping.store(true);
  s->s->join_all();
  delete s;
}

}  // extern "C"
