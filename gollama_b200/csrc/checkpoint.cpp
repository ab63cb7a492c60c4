// Checkpoint files, host side.
//
// Two formats:
//
//  - The reference's text checkpoint, written by Trainer.SaveCheckpoint
//    (pkg/train/trainer.go:554-584): a header of `key=value` lines
//    (GOLLAMA_CKPT, step, vocab_size, hidden_size, num_layers, num_heads,
//    intermediate_size), a `WEIGHTS` line, then one line per parameter in
//    Params() order holding each float32 as Go's fmt `%v` prints it followed
//    by one space.  The reference has no reader; the one here reads what the
//    writer (and therefore the reference) produces, so a text checkpoint
//    round-trips bit for bit (`%v` prints the shortest decimal that reads back
//    as the same float32).  Values may also be spelled as other plain
//    decimals ("0.50", "1E5"), each read as the nearest float32.
//
//  - A binary resume file holding what the text format leaves out: AdamW's
//    first and second moments and step counter, and the LR scheduler's step.
//    Layout (little-endian):
//        0  char[8]  "GLCSTATE"
//        8  u32      version (1)
//       12  u32      header bytes (80)
//       16  i64      trainer step (LRScheduler)
//       24  i64      AdamW step
//       32  i32 x 8  vocab, hidden, layers, heads, kv heads, intermediate,
//                    max_seq_len, semantics
//       64  i64      floats per arena (n)
//       72  u64      hash of bytes 0..71 and of the payload (below)
//       80  f32[n] parameters, f32[n] m, f32[n] v
//    The hash runs over the header's first 72 bytes, then the payload, as
//    64-bit words, h = (h ^ w) * P with the FNV-1a 64 offset basis and prime,
//    so a truncated or altered file (step counters included) is refused
//    before anything is written to the model.
//
// Both formats stream through fixed-size chunks, so saving or loading a model
// never holds more than a few chunks of host memory.  Nothing here touches the
// device: the trainer supplies and consumes the floats through callbacks.
#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "glc_internal.h"

namespace glc {

std::string& host_error() {
  thread_local std::string msg;
  return msg;
}

namespace {

int host_fail(int code, const std::string& msg) {
  host_error() = msg;
  return code;
}

constexpr int64_t kChunkFloats = int64_t(1) << 22;  // 16 MiB of float32 per chunk
constexpr uint64_t kHashBasis = 1469598103934665603ull;
constexpr uint64_t kHashPrime = 1099511628211ull;
constexpr char kStateMagic[8] = {'G', 'L', 'C', 'S', 'T', 'A', 'T', 'E'};
constexpr uint32_t kStateVersion = 1;
constexpr uint32_t kStateHeader = 80;

struct File {
  std::FILE* f = nullptr;
  ~File() {
    if (f) std::fclose(f);
  }
  bool close() {
    int rc = f ? std::fclose(f) : 0;
    f = nullptr;
    return rc == 0;
  }
};

// The header fields of the text format (trainer.go:566-573), in file order.
struct TextDims {
  const char* key;
  int value;
};

std::vector<TextDims> text_dims(const glc_train_config& cfg) {
  return {{"vocab_size", cfg.vocab_size},
          {"hidden_size", cfg.hidden_size},
          {"num_layers", cfg.num_layers},
          {"num_heads", cfg.num_heads},
          {"intermediate_size", cfg.intermediate_size}};
}

void hash_words(uint64_t& h, const void* p, size_t bytes) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  size_t i = 0;
  for (; i + 8 <= bytes; i += 8) {
    uint64_t w;
    std::memcpy(&w, b + i, 8);
    h = (h ^ w) * kHashPrime;
  }
  if (i < bytes) {  // a tail shorter than a word, zero-padded
    uint64_t w = 0;
    std::memcpy(&w, b + i, bytes - i);
    h = (h ^ w) * kHashPrime;
  }
}

}  // namespace

// ---------------------------------------------------------------- Go's %v
//
// fmt prints a float32 under %v as strconv.FormatFloat(float64(v), 'g', -1, 32):
// the shortest decimal digits d1..dn that read back as v, with decimal
// exponent x = (position of the decimal point) - 1.  For the shortest form
// %g switches at precision 6: the layout is scientific (d1[.d2..dn]e±XX, at
// least two exponent digits) when x < -4 or x >= 6, else positional with
// exactly as many fraction digits as the digits need.
// Infinities print with their sign ("+Inf", "-Inf"), NaN as "NaN", and the
// zero of either sign as "0" / "-0".  std::to_chars gives the same shortest
// digits (both pick, among the shortest round-tripping strings, the one
// closest to v).
int format_go_float32(float v, char* out) {
  char* p = out;
  if (std::isnan(v)) {
    std::memcpy(out, "NaN", 3);
    return 3;
  }
  if (std::signbit(v)) *p++ = '-';
  if (std::isinf(v)) {
    if (p == out) *p++ = '+';
    std::memcpy(p, "Inf", 3);
    return static_cast<int>(p + 3 - out);
  }
  if (v == 0.f) {
    *p++ = '0';
    return static_cast<int>(p - out);
  }
  // shortest digits in scientific form: d[.ddd]e[+-]XX
  char sci[32];
  auto r = std::to_chars(sci, sci + sizeof(sci), std::fabs(v), std::chars_format::scientific);
  char digits[16];
  int nd = 0;
  const char* q = sci;
  for (; q < r.ptr && *q != 'e'; ++q)
    if (*q != '.') digits[nd++] = *q;
  int x = 0;
  std::from_chars(q + 1 + (q[1] == '+'), r.ptr, x);
  if (x < -4 || x >= 6) {
    *p++ = digits[0];
    if (nd > 1) {
      *p++ = '.';
      for (int i = 1; i < nd; ++i) *p++ = digits[i];
    }
    *p++ = 'e';
    *p++ = x < 0 ? '-' : '+';
    int ax = x < 0 ? -x : x;
    if (ax < 10) *p++ = '0';
    auto e = std::to_chars(p, p + 4, ax);
    p = e.ptr;
    return static_cast<int>(p - out);
  }
  const int dp = x + 1;  // digits before the decimal point (may be <= 0)
  if (dp <= 0) {
    *p++ = '0';
  } else {
    for (int i = 0; i < dp; ++i) *p++ = i < nd ? digits[i] : '0';
  }
  if (nd > dp) {
    *p++ = '.';
    for (int i = dp; i < nd; ++i) *p++ = i < 0 ? '0' : digits[i];
  }
  return static_cast<int>(p - out);
}

// The inverse on one token: the strings above, and any other plain decimal
// (digits, at most one point, an optional exponent; a leading '-' only),
// rounded to the nearest float32.
bool parse_go_float32(const char* s, const char* e, float* v) {
  if (s >= e) return false;
  const size_t n = static_cast<size_t>(e - s);
  if (n == 3 && std::memcmp(s, "NaN", 3) == 0) {
    *v = std::nanf("");
    return true;
  }
  if (n == 4 && (s[0] == '+' || s[0] == '-') && std::memcmp(s + 1, "Inf", 3) == 0) {
    *v = s[0] == '-' ? -INFINITY : INFINITY;
    return true;
  }
  // digits, one optional '.', an optional exponent; a leading '-' only
  const char* q = s + (*s == '-');
  if (q >= e || !(*q >= '0' && *q <= '9')) return false;
  auto r = std::from_chars(s, e, *v, std::chars_format::general);
  return r.ec == std::errc() && r.ptr == e;
}

// ---------------------------------------------------------------- text writer

int ckpt_text_write(const char* path, int step, const glc_train_config& cfg, const std::vector<int64_t>& sizes,
                    const CkptFetch& fetch) {
  File f;
  f.f = std::fopen(path, "wb");
  if (!f.f) return host_fail(GLC_ERR_IO, std::string("checkpoint: cannot create ") + path + ": " + std::strerror(errno));
  std::string head = "GOLLAMA_CKPT\nstep=" + std::to_string(step) + "\n";
  for (const auto& d : text_dims(cfg)) head += std::string(d.key) + "=" + std::to_string(d.value) + "\n";
  head += "WEIGHTS\n";
  bool ok = std::fwrite(head.data(), 1, head.size(), f.f) == head.size();
  // Each chunk of floats is formatted by several threads into their own
  // buffers, then written in order (a float prints in at most 15 bytes plus
  // the separating space).
  const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<float> chunk(static_cast<size_t>(kChunkFloats));
  std::vector<std::string> parts(hw);
  int64_t off = 0;
  for (size_t pi = 0; pi < sizes.size() && ok; ++pi) {
    for (int64_t done = 0; done < sizes[pi] && ok;) {
      const int64_t n = std::min(kChunkFloats, sizes[pi] - done);
      if (!fetch(off + done, n, chunk.data()))
        return host_fail(GLC_ERR_CUDA, "checkpoint: reading the parameters from the device failed");
      const int nthreads = n >= 65536 ? static_cast<int>(hw) : 1;
      auto work = [&](int t) {
        const int64_t a = n * t / nthreads, b = n * (t + 1) / nthreads;
        std::string& s = parts[t];
        s.resize(static_cast<size_t>(b - a) * 16);
        char* w = s.data();
        for (int64_t i = a; i < b; ++i) {
          w += format_go_float32(chunk[i], w);
          *w++ = ' ';
        }
        s.resize(static_cast<size_t>(w - s.data()));
      };
      if (nthreads == 1) {
        work(0);
      } else {
        std::vector<std::thread> th;
        for (int t = 0; t < nthreads; ++t) th.emplace_back(work, t);
        for (auto& t : th) t.join();
      }
      for (int t = 0; t < nthreads && ok; ++t) ok = std::fwrite(parts[t].data(), 1, parts[t].size(), f.f) == parts[t].size();
      done += n;
    }
    ok = ok && std::fputc('\n', f.f) != EOF;
    off += sizes[pi];
  }
  if (!f.close() || !ok) return host_fail(GLC_ERR_IO, std::string("checkpoint: write failed on ") + path);
  return GLC_OK;
}

// ---------------------------------------------------------------- text reader

namespace {

// Buffered reader over a FILE*: values are parsed in place from the buffer.
struct Reader {
  std::FILE* f;
  std::vector<char> buf = std::vector<char>(size_t(1) << 22);
  size_t pos = 0, len = 0;
  bool eof = false;
  // Keeps the unread bytes and appends more; false at the end of the file.
  bool refill() {
    if (eof) return false;
    if (pos > 0) {
      std::memmove(buf.data(), buf.data() + pos, len - pos);
      len -= pos;
      pos = 0;
    }
    if (len == buf.size()) return false;  // a token longer than the buffer
    const size_t got = std::fread(buf.data() + len, 1, buf.size() - len, f);
    len += got;
    if (got == 0) eof = true;
    return got > 0;
  }
  int get() {
    if (pos == len && !refill()) return EOF;
    return static_cast<unsigned char>(buf[pos++]);
  }
  // The next token up to ' ' or '\n' (not included) as [*s, *e); *term is
  // the terminator, EOF at the end of the file.  The token is valid until the
  // next call.  False when a token exceeds max_len bytes.
  bool token(const char** s, const char** e, int* term, size_t max_len) {
    for (size_t scan = pos;;) {
      const char* b = buf.data();
      for (; scan < len; ++scan) {
        if (b[scan] == ' ' || b[scan] == '\n') {
          *s = b + pos;
          *e = b + scan;
          *term = b[scan];
          pos = scan + 1;
          return scan - (*s - b) <= max_len;
        }
        if (scan - pos > max_len) return false;
      }
      const size_t have = len - pos;
      if (!refill()) {
        *s = buf.data() + pos;
        *e = buf.data() + len;
        *term = EOF;
        pos = len;
        return have <= max_len;
      }
      scan = pos + have;
    }
  }
  bool line(std::string& out, size_t max_len) {
    out.clear();
    for (;;) {
      int c = get();
      if (c == '\n') return true;
      if (c == EOF || out.size() >= max_len) return false;
      out.push_back(static_cast<char>(c));
    }
  }
};

// One slice of a block of the WEIGHTS section, parsed by one thread: its
// values in order, after how many values each line ended, and the first
// malformed token with the values and line ends before it.  A line is
// "v v ... v \n": the token before each '\n' is empty.
struct Slice {
  std::vector<float> vals;
  std::vector<int64_t> ends;
  bool bad = false;
  int64_t bad_at = 0;
  size_t bad_ends = 0;
  std::string bad_tok;
};

// [a, b) starts at a token and ends just after a separator.
void parse_slice(const char* a, const char* b, Slice* s) {
  s->vals.clear();
  s->ends.clear();
  s->bad = false;
  s->vals.reserve(static_cast<size_t>(b - a) / 10 + 1);
  const char* t = a;
  for (const char* p = a; p < b; ++p) {
    const char c = *p;
    if (c != ' ' && c != '\n') continue;
    if (c == '\n' && p == t) {
      s->ends.push_back(static_cast<int64_t>(s->vals.size()));
    } else {
      float v;
      // a value ends with a space, never with the line
      if (c == '\n' || p - t > 32 || !parse_go_float32(t, p, &v)) {
        s->bad = true;
        s->bad_at = static_cast<int64_t>(s->vals.size());
        s->bad_ends = s->ends.size();
        s->bad_tok.assign(t, std::min(p, t + 40));
        if (c == '\n') s->bad_tok += "\\n";
        return;
      }
      s->vals.push_back(v);
    }
    t = p + 1;
  }
}

bool parse_int_field(const std::string& line, const char* key, long long* v) {
  const size_t k = std::strlen(key);
  if (line.size() <= k + 1 || line.compare(0, k, key) != 0 || line[k] != '=') return false;
  const char* s = line.data() + k + 1;
  const char* e = line.data() + line.size();
  auto r = std::from_chars(s, e, *v);
  return r.ec == std::errc() && r.ptr == e;
}

}  // namespace

int ckpt_text_read(const char* path, const glc_train_config& cfg, const std::vector<int64_t>& sizes, int* step,
                   const CkptStore& store) {
  File f;
  f.f = std::fopen(path, "rb");
  if (!f.f) return host_fail(GLC_ERR_IO, std::string("checkpoint: cannot open ") + path + ": " + std::strerror(errno));
  Reader rd{f.f};
  std::string line;
  const std::string where = std::string("checkpoint ") + path + ": ";
  if (!rd.line(line, 64) || line != "GOLLAMA_CKPT") return host_fail(GLC_ERR_IO, where + "not a GOLLAMA_CKPT file");
  long long st = 0;
  if (!rd.line(line, 64) || !parse_int_field(line, "step", &st) || st < 0 || st > INT32_MAX)
    return host_fail(GLC_ERR_IO, where + "bad step line");
  for (const auto& d : text_dims(cfg)) {
    long long v = 0;
    if (!rd.line(line, 64) || !parse_int_field(line, d.key, &v))
      return host_fail(GLC_ERR_IO, where + "bad " + d.key + " line");
    if (v != d.value)
      return host_fail(GLC_ERR_INVALID, where + d.key + "=" + std::to_string(v) + " but the model has " +
                                            std::to_string(d.value));
  }
  if (!rd.line(line, 64) || line != "WEIGHTS") return host_fail(GLC_ERR_IO, where + "missing WEIGHTS line");
  // The WEIGHTS section in blocks: each block up to its last separator is
  // cut at separators into one slice per thread, the slices are parsed in
  // parallel, then checked and stored in file order.
  const unsigned nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<char> blk(size_t(1) << 26);
  size_t have = rd.len - rd.pos;
  std::memcpy(blk.data(), rd.buf.data() + rd.pos, have);
  std::vector<Slice> slices(nth);
  const size_t np = sizes.size();
  size_t pi = 0;        // parameter being read
  int64_t in_param = 0;  // its values so far
  int64_t off = 0;       // arena offset of the next value
  const auto holds = [&](int64_t k) {
    return where + "parameter " + std::to_string(pi) + " holds " + std::to_string(k) + " values, the model " +
           std::to_string(sizes[pi]);
  };
  // Checks the line ends and values of a slice (up to n_ends ends and n_vals
  // values) against the parameter sizes; returns 0 or the error.
  const auto check = [&](const Slice& sl, size_t n_ends, int64_t n_vals) -> int {
    int64_t prev = 0;
    for (size_t k = 0; k <= n_ends; ++k) {
      const int64_t upto = k < n_ends ? sl.ends[k] : n_vals;
      const int64_t cnt = upto - prev;
      prev = upto;
      if (k == n_ends && cnt == 0) break;
      if (pi >= np) return host_fail(GLC_ERR_INVALID, where + "more parameters than the model has");
      in_param += cnt;
      if (in_param > sizes[pi]) return host_fail(GLC_ERR_INVALID, holds(in_param) + " (or more)");
      if (k < n_ends) {
        if (in_param != sizes[pi]) return host_fail(GLC_ERR_INVALID, holds(in_param));
        ++pi;
        in_param = 0;
      }
    }
    return GLC_OK;
  };
  for (bool at_eof = false; !(at_eof && have == 0);) {
    if (!at_eof) {
      const size_t got = std::fread(blk.data() + have, 1, blk.size() - have, f.f);
      have += got;
      at_eof = got == 0 || std::feof(f.f);
    }
    size_t last = have;  // one past the last separator
    while (last > 0 && blk[last - 1] != ' ' && blk[last - 1] != '\n') --last;
    if (last == 0) {
      if (at_eof && have > 0)
        return host_fail(GLC_ERR_IO, where + "truncated: the file ends inside a value");
      if (have == blk.size()) return host_fail(GLC_ERR_IO, where + "malformed: no separator in a block");
      if (at_eof) break;
      continue;
    }
    // slice boundaries, each just after a separator
    std::vector<size_t> cut(nth + 1, last);
    cut[0] = 0;
    for (unsigned t = 1; t < nth; ++t) {
      size_t c = std::max(cut[t - 1], last * t / nth);
      while (c < last && c > 0 && blk[c - 1] != ' ' && blk[c - 1] != '\n') ++c;
      cut[t] = c;
    }
    if (last < 65536) {
      for (unsigned t = 1; t < nth; ++t) cut[t] = last;
    }
    std::vector<std::thread> th;
    for (unsigned t = 1; t < nth; ++t)
      if (cut[t] < cut[t + 1]) th.emplace_back(parse_slice, blk.data() + cut[t], blk.data() + cut[t + 1], &slices[t]);
    parse_slice(blk.data() + cut[0], blk.data() + cut[1], &slices[0]);
    for (auto& x : th) x.join();
    for (unsigned t = 0; t < nth; ++t) {
      if (cut[t] >= cut[t + 1]) continue;
      const Slice& sl = slices[t];
      const size_t n_ends = sl.bad ? sl.bad_ends : sl.ends.size();
      const int64_t n_vals = sl.bad ? sl.bad_at : static_cast<int64_t>(sl.vals.size());
      int rc = check(sl, n_ends, n_vals);
      if (rc) return rc;
      if (sl.bad)
        return host_fail(GLC_ERR_IO, where + "malformed value '" + sl.bad_tok + "' in parameter " + std::to_string(pi));
      if (n_vals > 0 && !store(off, n_vals, sl.vals.data()))
        return host_fail(GLC_ERR_CUDA, "checkpoint: writing the parameters to the device failed");
      off += n_vals;
    }
    std::memmove(blk.data(), blk.data() + last, have - last);
    have -= last;
  }
  if (pi != np || in_param != 0)
    return host_fail(GLC_ERR_IO, where + "truncated: the file ends in parameter " + std::to_string(pi) + " of " +
                                     std::to_string(np));
  *step = static_cast<int>(st);
  return GLC_OK;
}

// ---------------------------------------------------------------- binary state

namespace {

void put32(unsigned char* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = static_cast<unsigned char>(v >> (8 * i));
}
void put64(unsigned char* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = static_cast<unsigned char>(v >> (8 * i));
}
uint32_t get32(const unsigned char* p) {
  uint32_t v = 0;
  for (int i = 0; i < 4; ++i) v |= static_cast<uint32_t>(p[i]) << (8 * i);
  return v;
}
uint64_t get64(const unsigned char* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(p[i]) << (8 * i);
  return v;
}

std::array<int32_t, 8> state_dims(const glc_train_config& c) {
  const int kv = c.semantics == GLC_SEMANTICS_LLAMA && c.num_kv_heads > 0 ? c.num_kv_heads : c.num_heads;
  return {c.vocab_size, c.hidden_size, c.num_layers, c.num_heads, kv, c.intermediate_size, c.max_seq_len, c.semantics};
}

const char* kDimNames[8] = {"vocab_size",        "hidden_size", "num_layers", "num_heads",
                            "num_kv_heads",      "intermediate_size", "max_seq_len", "semantics"};

}  // namespace

int state_write(const char* path, const StateInfo& info, const glc_train_config& cfg, int64_t n,
                const StateFetch& fetch) {
  File f;
  f.f = std::fopen(path, "wb");
  if (!f.f) return host_fail(GLC_ERR_IO, std::string("state: cannot create ") + path + ": " + std::strerror(errno));
  unsigned char head[kStateHeader] = {};
  std::memcpy(head, kStateMagic, 8);
  put32(head + 8, kStateVersion);
  put32(head + 12, kStateHeader);
  put64(head + 16, static_cast<uint64_t>(info.step));
  put64(head + 24, static_cast<uint64_t>(info.adam_step));
  const auto dims = state_dims(cfg);
  for (int i = 0; i < 8; ++i) put32(head + 32 + 4 * i, static_cast<uint32_t>(dims[i]));
  put64(head + 64, static_cast<uint64_t>(n));
  // the hash goes in last: write a placeholder, then seek back
  bool ok = std::fwrite(head, 1, kStateHeader, f.f) == kStateHeader;
  uint64_t h = kHashBasis;
  hash_words(h, head, 72);
  std::vector<float> chunk(static_cast<size_t>(std::min<int64_t>(kChunkFloats, std::max<int64_t>(n, 1))));
  for (int arena = 0; arena < 3 && ok; ++arena) {
    for (int64_t off = 0; off < n && ok; off += kChunkFloats) {
      const int64_t k = std::min(kChunkFloats, n - off);
      if (!fetch(arena, off, k, chunk.data()))
        return host_fail(GLC_ERR_CUDA, "state: reading the model from the device failed");
      hash_words(h, chunk.data(), sizeof(float) * static_cast<size_t>(k));
      ok = std::fwrite(chunk.data(), sizeof(float), static_cast<size_t>(k), f.f) == static_cast<size_t>(k);
    }
  }
  put64(head + 72, h);
  ok = ok && std::fseek(f.f, 72, SEEK_SET) == 0 && std::fwrite(head + 72, 1, 8, f.f) == 8;
  if (!f.close() || !ok) return host_fail(GLC_ERR_IO, std::string("state: write failed on ") + path);
  return GLC_OK;
}

int state_read(const char* path, const glc_train_config& cfg, int64_t n, StateInfo* info, const StateStore& store) {
  File f;
  f.f = std::fopen(path, "rb");
  if (!f.f) return host_fail(GLC_ERR_IO, std::string("state: cannot open ") + path + ": " + std::strerror(errno));
  const std::string where = std::string("state ") + path + ": ";
  unsigned char head[kStateHeader];
  if (std::fread(head, 1, kStateHeader, f.f) != kStateHeader || std::memcmp(head, kStateMagic, 8) != 0)
    return host_fail(GLC_ERR_IO, where + "not a GLCSTATE file");
  if (get32(head + 8) != kStateVersion || get32(head + 12) != kStateHeader)
    return host_fail(GLC_ERR_IO, where + "unknown version " + std::to_string(get32(head + 8)));
  const auto dims = state_dims(cfg);
  for (int i = 0; i < 8; ++i) {
    const int32_t v = static_cast<int32_t>(get32(head + 32 + 4 * i));
    if (v != dims[i])
      return host_fail(GLC_ERR_INVALID, where + kDimNames[i] + "=" + std::to_string(v) + " but the model has " +
                                            std::to_string(dims[i]));
  }
  if (static_cast<int64_t>(get64(head + 64)) != n)
    return host_fail(GLC_ERR_INVALID, where + "holds " + std::to_string(get64(head + 64)) +
                                          " floats per arena, the model " + std::to_string(n));
  const int64_t st = static_cast<int64_t>(get64(head + 16)), ast = static_cast<int64_t>(get64(head + 24));
  if (st < 0 || st > INT32_MAX || ast < 0 || ast > INT32_MAX) return host_fail(GLC_ERR_IO, where + "bad step counters");
  // size, then hash, before anything reaches the model
  if (std::fseek(f.f, 0, SEEK_END) != 0) return host_fail(GLC_ERR_IO, where + "cannot seek");
  const long long bytes = std::ftell(f.f);
  if (bytes != static_cast<long long>(kStateHeader) + 12ll * n)
    return host_fail(GLC_ERR_IO, where + "size " + std::to_string(bytes) + " bytes, expected " +
                                     std::to_string(kStateHeader + 12ll * n) + " (truncated or padded)");
  std::vector<float> chunk(static_cast<size_t>(std::min<int64_t>(kChunkFloats, std::max<int64_t>(n, 1))));
  for (int pass = 0; pass < 2; ++pass) {
    if (std::fseek(f.f, kStateHeader, SEEK_SET) != 0) return host_fail(GLC_ERR_IO, where + "cannot seek");
    uint64_t h = kHashBasis;
    hash_words(h, head, 72);
    for (int arena = 0; arena < 3; ++arena) {
      for (int64_t off = 0; off < n; off += kChunkFloats) {
        const int64_t k = std::min(kChunkFloats, n - off);
        if (std::fread(chunk.data(), sizeof(float), static_cast<size_t>(k), f.f) != static_cast<size_t>(k))
          return host_fail(GLC_ERR_IO, where + "short read");
        if (pass == 0) {
          hash_words(h, chunk.data(), sizeof(float) * static_cast<size_t>(k));
        } else if (!store(arena, off, k, chunk.data())) {
          return host_fail(GLC_ERR_CUDA, "state: writing the model to the device failed");
        }
      }
    }
    if (pass == 0 && h != get64(head + 72)) return host_fail(GLC_ERR_IO, where + "hash mismatch (corrupt file)");
  }
  info->step = static_cast<int>(st);
  info->adam_step = static_cast<int>(ast);
  return GLC_OK;
}

}  // namespace glc

// ---------------------------------------------------------------- C ABI (host buffers only)

using glc::host_fail;

extern "C" {

int glc_checkpoint_write(const char* path, int step, const glc_train_config* cfg, const float* params, int64_t n) {
  if (!path || !cfg || !params || step < 0) return host_fail(GLC_ERR_INVALID, "checkpoint: bad arguments");
  std::vector<int64_t> sizes;
  if (!glc::param_sizes(*cfg, &sizes)) return host_fail(GLC_ERR_INVALID, "checkpoint: inconsistent configuration");
  int64_t total = 0;
  for (int64_t s : sizes) total += s;
  if (n != total) return host_fail(GLC_ERR_INVALID, "checkpoint: n is not the model's parameter count");
  return glc::ckpt_text_write(path, step, *cfg, sizes, [&](int64_t off, int64_t k, float* dst) {
    std::memcpy(dst, params + off, sizeof(float) * static_cast<size_t>(k));
    return true;
  });
}

int glc_checkpoint_read(const char* path, const glc_train_config* cfg, int* step, float* params, int64_t n) {
  if (!path || !cfg || !step || !params) return host_fail(GLC_ERR_INVALID, "checkpoint: bad arguments");
  std::vector<int64_t> sizes;
  if (!glc::param_sizes(*cfg, &sizes)) return host_fail(GLC_ERR_INVALID, "checkpoint: inconsistent configuration");
  int64_t total = 0;
  for (int64_t s : sizes) total += s;
  if (n != total) return host_fail(GLC_ERR_INVALID, "checkpoint: n is not the model's parameter count");
  return glc::ckpt_text_read(path, *cfg, sizes, step, [&](int64_t off, int64_t k, const float* src) {
    std::memcpy(params + off, src, sizeof(float) * static_cast<size_t>(k));
    return true;
  });
}

int glc_state_write(const char* path, const glc_train_config* cfg, int step, int adam_step, const float* params,
                    const float* m, const float* v, int64_t n) {
  if (!path || !cfg || !params || !m || !v || n < 0 || step < 0 || adam_step < 0)
    return host_fail(GLC_ERR_INVALID, "state: bad arguments");
  const float* arenas[3] = {params, m, v};
  return glc::state_write(path, glc::StateInfo{step, adam_step}, *cfg, n,
                          [&](int a, int64_t off, int64_t k, float* dst) {
                            std::memcpy(dst, arenas[a] + off, sizeof(float) * static_cast<size_t>(k));
                            return true;
                          });
}

int glc_state_read(const char* path, const glc_train_config* cfg, int* step, int* adam_step, float* params, float* m,
                   float* v, int64_t n) {
  if (!path || !cfg || !step || !adam_step || !params || !m || !v || n < 0)
    return host_fail(GLC_ERR_INVALID, "state: bad arguments");
  float* arenas[3] = {params, m, v};
  glc::StateInfo info{};
  int rc = glc::state_read(path, *cfg, n, &info, [&](int a, int64_t off, int64_t k, const float* src) {
    std::memcpy(arenas[a] + off, src, sizeof(float) * static_cast<size_t>(k));
    return true;
  });
  if (rc) return rc;
  *step = info.step;
  *adam_step = info.adam_step;
  return GLC_OK;
}

}  // extern "C"
