// Weight manifest: the tensor index of an exported engine (convert/export_engine.py:29-34, 83-85) and the
// name -> (shard, offset) resolution of the engine's w(name) (web/public/engine/engine.js:175-180).
//
// The manifest is the JSON the exporter writes: "shards": [{"path", "start", "bytes"}, ...] (shards of at
// most 512 MB, split only between tensors, laid out back to back from global offset 0), and "tensors":
// {name: {"offset", "bytes", "dtype", "shape", "N", "K"}} with global, 256-byte aligned offsets; a
// quantised projection `p` is the pair `p.q` (uint8 [N][K/32][16], N padded to 64 rows, with N and K)
// and `p.s` (float16 [N][K/32]). Host code only: parsing and lookups allocate host memory, never device
// memory; s4_weight_upload_named hands the resolved ranges to the regular upload entry points.
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"

struct s4_manifest {
  struct Shard {
    std::string path;
    long long start = 0, bytes = 0;
  };
  struct Tensor {
    long long offset = -1, bytes = -1;
    std::string dtype;
    std::vector<long long> shape;
    long long N = -1, K = -1;
  };
  std::vector<Shard> shards;
  std::unordered_map<std::string, Tensor> tensors;
};

namespace {

// A small recursive-descent reader for the manifest's JSON (objects, arrays, strings, integers; other
// values are skipped).
struct Reader {
  const char* p;
  const char* end;
  std::string why;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(char c) {
    ws();
    if (p < end && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool peek(char c) {
    ws();
    return p < end && *p == c;
  }
  bool str(std::string& out) {
    ws();
    if (p >= end || *p != '"') return false;
    ++p;
    out.clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return false;
        switch (*p) {
          case 'n': out.push_back('\n'); break;
          case 't': out.push_back('\t'); break;
          case 'r': out.push_back('\r'); break;
          case 'b': out.push_back('\b'); break;
          case 'f': out.push_back('\f'); break;
          case 'u': {  // \uXXXX: ASCII only (tensor and shard names are ASCII)
            if (end - p < 5) return false;
            char hex[5] = {p[1], p[2], p[3], p[4], 0};
            const long v = strtol(hex, nullptr, 16);
            if (v < 0 || v > 0x7f) return false;
            out.push_back((char)v);
            p += 4;
            break;
          }
          default: out.push_back(*p);
        }
        ++p;
        continue;
      }
      out.push_back(*p++);
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool num(long long& v) {
    ws();
    char* e = nullptr;
    errno = 0;
    const long long r = strtoll(p, &e, 10);
    if (e == p || errno) return false;
    // an integer field must not carry a fraction or exponent
    if (e < end && (*e == '.' || *e == 'e' || *e == 'E')) return false;
    v = r;
    p = e;
    return true;
  }
  bool skip() {
    ws();
    if (p >= end) return false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = (*p == '{') ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (lit(close)) return true;
      for (;;) {
        if (obj) {
          std::string k;
          if (!str(k) || !lit(':')) return false;
        }
        if (!skip()) return false;
        if (lit(close)) return true;
        if (!lit(',')) return false;
      }
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
  // Calls f(key) for every member of an object; f must consume the value.
  template <class F>
  bool object(F f) {
    if (!lit('{')) return false;
    if (lit('}')) return true;
    for (;;) {
      std::string k;
      if (!str(k) || !lit(':')) return false;
      if (!f(k)) return false;
      if (lit('}')) return true;
      if (!lit(',')) return false;
    }
  }
  template <class F>
  bool array(F f) {
    if (!lit('[')) return false;
    if (lit(']')) return true;
    for (;;) {
      if (!f()) return false;
      if (lit(']')) return true;
      if (!lit(',')) return false;
    }
  }
};

bool parse_manifest(const char* text, size_t len, s4_manifest& m, std::string& why) {
  Reader r{text, text + len, {}};
  bool have_tensors = false;
  const bool ok = r.object([&](const std::string& key) {
    if (key == "shards") {
      return r.array([&] {
        s4_manifest::Shard s;
        const bool okk = r.object([&](const std::string& k) {
          if (k == "path") return r.str(s.path);
          if (k == "start") return r.num(s.start);
          if (k == "bytes") return r.num(s.bytes);
          return r.skip();
        });
        if (okk) m.shards.push_back(s);
        return okk;
      });
    }
    if (key == "tensors") {
      have_tensors = true;
      return r.object([&](const std::string& name) {
        s4_manifest::Tensor t;
        const bool okk = r.object([&](const std::string& k) {
          if (k == "offset") return r.num(t.offset);
          if (k == "bytes") return r.num(t.bytes);
          if (k == "dtype") return r.str(t.dtype);
          if (k == "N") return r.num(t.N);
          if (k == "K") return r.num(t.K);
          if (k == "shape")
            return r.array([&] {
              long long v;
              if (!r.num(v)) return false;
              t.shape.push_back(v);
              return true;
            });
          return r.skip();
        });
        if (!okk) return false;
        if (t.offset < 0 || t.bytes < 0) {
          why = "tensor " + name + " lacks offset or bytes";
          return false;
        }
        m.tensors[name] = t;
        return true;
      });
    }
    return r.skip();
  });
  if (!ok) {
    if (why.empty()) why = "malformed JSON near byte " + std::to_string(r.p - text);
    return false;
  }
  if (!have_tensors) return why = "no \"tensors\" index", false;
  if (m.shards.empty()) return why = "no \"shards\" list", false;
  for (const auto& s : m.shards)
    if (s.start < 0 || s.bytes < 0) return why = "shard " + s.path + " has a negative start or size", false;
  return true;
}

// w(name): the shard holding the tensor's first byte and the offset inside it; the tensor must end
// inside that shard too (the exporter splits shards only between tensors).
int resolve(const s4_manifest* m, const char* name, const s4_manifest::Tensor** tout, int* shard, size_t* offset) {
  auto it = m->tensors.find(name);
  if (it == m->tensors.end()) {
    std::string msg = std::string("no tensor ") + name;  // engine.js:177
    return s4::record_error(S4_ERR_INVALID, msg.c_str());
  }
  const s4_manifest::Tensor& t = it->second;
  for (int i = 0; i < (int)m->shards.size(); ++i) {
    const auto& s = m->shards[i];
    if (t.offset >= s.start && t.offset < s.start + s.bytes) {
      if (t.offset + t.bytes > s.start + s.bytes) {
        std::string msg = std::string("tensor ") + name + " runs past the end of shard " + s.path;
        return s4::record_error(S4_ERR_INVALID, msg.c_str());
      }
      *tout = &t;
      *shard = i;
      *offset = (size_t)(t.offset - s.start);
      return S4_OK;
    }
  }
  std::string msg = std::string("tensor ") + name + " lies in no shard";
  return s4::record_error(S4_ERR_INVALID, msg.c_str());
}

}  // namespace

extern "C" {

int s4_manifest_open(const char* json, s4_manifest** out) {
  if (!json || !out) return s4::record_error(S4_ERR_INVALID, "s4_manifest_open: NULL argument");
  *out = nullptr;
  s4_manifest* m = new (std::nothrow) s4_manifest();
  if (!m) return s4::record_error(S4_ERR_NOMEM, "s4_manifest_open: out of host memory");
  std::string why;
  bool ok = false;
  try {
    ok = parse_manifest(json, strlen(json), *m, why);
  } catch (const std::bad_alloc&) {
    delete m;
    return s4::record_error(S4_ERR_NOMEM, "s4_manifest_open: out of host memory");
  }
  if (!ok) {
    delete m;
    why = "s4_manifest_open: " + why;
    return s4::record_error(S4_ERR_INVALID, why.c_str());
  }
  *out = m;
  return S4_OK;
}

int s4_manifest_free(s4_manifest* m) {
  delete m;
  return S4_OK;
}

int s4_manifest_counts(const s4_manifest* m, int* nshards, int* ntensors) {
  if (!m) return s4::record_error(S4_ERR_INVALID, "s4_manifest_counts: NULL manifest");
  if (nshards) *nshards = (int)m->shards.size();
  if (ntensors) *ntensors = (int)m->tensors.size();
  return S4_OK;
}

int s4_manifest_shard(const s4_manifest* m, int i, const char** path, size_t* bytes) {
  if (!m) return s4::record_error(S4_ERR_INVALID, "s4_manifest_shard: NULL manifest");
  if (i < 0 || i >= (int)m->shards.size()) return s4::record_error(S4_ERR_INVALID, "s4_manifest_shard: index out of range");
  if (path) *path = m->shards[i].path.c_str();
  if (bytes) *bytes = (size_t)m->shards[i].bytes;
  return S4_OK;
}

int s4_manifest_tensor(const s4_manifest* m, const char* name, int* shard, size_t* offset, size_t* bytes, int* N,
                       int* K) {
  if (!m || !name) return s4::record_error(S4_ERR_INVALID, "s4_manifest_tensor: NULL argument");
  const s4_manifest::Tensor* t = nullptr;
  int sh = -1;
  size_t off = 0;
  const int rc = resolve(m, name, &t, &sh, &off);
  if (rc != S4_OK) return rc;
  if (shard) *shard = sh;
  if (offset) *offset = off;
  if (bytes) *bytes = (size_t)t->bytes;
  if (N) *N = t->N > INT32_MAX ? -1 : (int)t->N;
  if (K) *K = t->K > INT32_MAX ? -1 : (int)t->K;
  return S4_OK;
}

int s4_weight_upload_named(s4_ctx* ctx, const s4_manifest* m, const void* const* shards, const char* name,
                           uint32_t flags, s4_weight** out) {
  if (!ctx || !m || !shards || !name || !out) return s4::record_error(S4_ERR_INVALID, "s4_weight_upload_named: NULL argument");
  if (flags & ~S4_UPLOAD_DEVICE) return s4::record_error(S4_ERR_INVALID, "s4_weight_upload_named: unknown flags");
  const std::string qn = std::string(name) + ".q", sn = std::string(name) + ".s";
  const s4_manifest::Tensor *tq = nullptr, *ts = nullptr;
  int shq = -1, shs = -1;
  size_t oq = 0, os = 0;
  int rc = resolve(m, qn.c_str(), &tq, &shq, &oq);
  if (rc == S4_OK) rc = resolve(m, sn.c_str(), &ts, &shs, &os);
  if (rc != S4_OK) return rc;
  std::string bad;
  if (tq->N < 1 || tq->K < 32 || tq->K % 32 || tq->N > INT32_MAX || tq->K > INT32_MAX)
    bad = qn + " lacks a valid N and K";
  else if (tq->dtype != "uint8" || tq->bytes != tq->N * (tq->K / 32) * 16)
    bad = qn + " is not uint8 [N][K/32][16]";
  else if (ts->dtype != "float16" || ts->bytes != tq->N * (tq->K / 32) * 2)
    bad = sn + " is not float16 [N][K/32]";
  else if (!shards[shq] || !shards[shs])
    bad = std::string("shard ") + m->shards[shq].path + " or " + m->shards[shs].path + " has no buffer";
  if (!bad.empty()) {
    bad = "s4_weight_upload_named: " + bad;
    return s4::record_error(S4_ERR_INVALID, bad.c_str());
  }
  const uint8_t* q = static_cast<const uint8_t*>(shards[shq]) + oq;
  const uint8_t* s = static_cast<const uint8_t*>(shards[shs]) + os;
  const int N = (int)tq->N, K = (int)tq->K;
  if (flags & S4_UPLOAD_DEVICE) return s4_weight_upload_device(ctx, q, s, N, K, 0, out);
  return s4_weight_upload(ctx, q, reinterpret_cast<const uint16_t*>(s), N, K, 0, out);
}

}  // extern "C"
