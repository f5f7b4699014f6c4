// C ABI of libs4mm.so: context, weight handles, dispatcher, launches. Declarations and the
// reference interfaces each entry point replaces are in include/s4mm.h.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include <sys/types.h>

#include "../../include/s4mm.h"
#include "common.cuh"
#include "internal.h"

using s4::Bucket;
using s4::DeviceGuard;

namespace s4 {
cudaError_t launch_repack(const uint8_t* packed, const __half* scales, uint32_t* wq, __half* ws, int N, int K,
                          int nblk, int ktiles, int sm_count, cudaStream_t stream, int glu_I);
cudaError_t launch_gemv(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, __half* y,
                        uint32_t* err, int M, int N, int K, int nblk, int ktiles, int token0, int groups, int split,
                        int sm_count, cudaStream_t stream, bool pdl, int glu, const uint8_t* wq2);
cudaError_t launch_repack2(const uint32_t* q, int N, int K, int nblk, int ktiles, uint8_t* out, int sm_count,
                           cudaStream_t stream);
int gemv_max_split();
int gemv_max_tokens();
cudaError_t launch_silu_mul(const __half* big, __half* mid, int M, int I, int sm_count, cudaStream_t stream);
cudaError_t launch_silu_mul_gather(const __half* big, int M, int Is, __half* const* dst, int ndst, int64_t ldd, int col0,
                                   int sm_count, cudaStream_t stream);
cudaError_t launch_wire_scales(const uint8_t* wire, int N, int G, const double* pow_table, uint16_t* out, int sms,
                               cudaStream_t stream);
cudaError_t launch_transcode(const uint32_t* q, const __half* scales, const __half* bias, int N, int K, int bits,
                             int group, uint8_t* packed4, __half* scales32, __half* bias32, int sm_count,
                             cudaStream_t stream);
cudaError_t launch_fwht(__half* a, int64_t blocks, int n, cudaStream_t stream);
cudaError_t launch_add_rmsnorm(float* x, const __half* y, const float* w, int M, int D, float eps, __half* h,
                               cudaStream_t stream, const uint32_t* wait_flags, int wait_n, uint32_t* err);
cudaError_t launch_peer_signal(uint32_t* const* flags, int nranks, int rank, cudaStream_t stream, bool pdl);
cudaError_t launch_peer_barrier(uint32_t* const* flags, int nranks, int rank, uint32_t epoch, uint32_t* err,
                                cudaStream_t stream);
cudaError_t launch_tc_gemm_ex(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, int64_t ldx,
                              __half* const* ydst,
                              int ndst, int64_t ldy, int ycol0, float* partials, uint32_t* tickets, int max_tickets,
                              uint32_t* err, int M, int N, int K, int nblk, int ktiles, int tile_n, int grid,
                              cudaStream_t stream, bool pdl, bool ticket_fixup, int glu, float* resid,
                              int64_t ldr, float* ssp, int64_t ldss, const uint32_t* wait_flags, int wait_n);
cudaError_t launch_rmsnorm_from_sums(const float* x, const float* ssp, int64_t ldss, const float* w, int M, int D,
                                     float eps, __half* h, cudaStream_t stream, bool pdl);
int chain_create(s4_ctx* ctx, int nops, const s4_weight* const* w, const void* const* x, void* const* y, const int* M,
                 const int* dep, s4_chain** out, const char** why);
cudaError_t chain_launch(s4_chain* c, uint32_t* err, cudaStream_t stream, bool cooperative);
void chain_destroy(s4_chain* c);
int chain_info(const s4_chain* c, int* grid, int* slots, int* smem);
bool tc_available();
size_t tc_partials_bytes(int max_grid);
cudaError_t launch_tc_gemm(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, __half* y,
                           float* partials, uint32_t* tickets, int max_tickets, uint32_t* err, int M, int N, int K,
                           int nblk, int ktiles, int tile_n, int grid, cudaStream_t stream, bool pdl,
                           bool ticket_fixup, int glu);
}  // namespace s4

namespace {

constexpr int kMaxTickets = 1 << 16;  // n-blocks per weight: N <= 8,388,608
// s4_matmul_add_rmsnorm's sums of squares: (N / 32) x rows per launch (16384 rows at N = 2048)
constexpr size_t kNormSums = 1u << 20;
constexpr int kGemvMaxM = 16;  // tokens one GEMV launch covers (two 8-token mma column groups)

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

}  // namespace

namespace s4 {
int record_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}
}  // namespace s4

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  return fail(S4_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace

namespace {

std::vector<Bucket> fallback_table() {
  // GEMV up to 16 tokens; tcgen05 GEMM above when the kernel is built in, else repeated GEMV
  // launches of 16 tokens.
  std::vector<Bucket> t;
  t.push_back({kGemvMaxM, S4_FAMILY_GEMV, 0, 0});
  t.push_back({INT_MAX, s4::tc_available() ? S4_FAMILY_TC : S4_FAMILY_GEMV, 0, 0});
  return t;
}

bool parse_table(const char* text, std::vector<Bucket>& out, std::string& why);

// The built-in M-bucket table (replaces engine.js:17-33): the measured table tune.py wrote into
// dispatch_table.inc, else the fallback above. Environment S4_TABLE=fallback selects the fallback.
std::vector<Bucket> default_table() {
#if __has_include("dispatch_table.inc")
#include "dispatch_table.inc"
  const char* env = getenv("S4_TABLE");
  if (!(env && strcmp(env, "fallback") == 0)) {
    std::vector<Bucket> t;
    std::string why;
    if (parse_table(kDispatchTableJson, t, why)) return t;
  }
#endif
  return fallback_table();
}

// The first bucket whose max_m covers M and whose K / N (when given) match the weight.
Bucket choose(const s4_ctx* ctx, int M, int N, int K) {
  if (ctx->forced.family != S4_FAMILY_AUTO) return ctx->forced;
  for (const Bucket& b : ctx->table)
    if (M <= b.max_m && (b.K == 0 || b.K == K) && (b.N == 0 || b.N == N)) return b;
  return ctx->table.empty() ? Bucket{INT_MAX, S4_FAMILY_GEMV, 0, 0} : ctx->table.back();
}

// ---- a minimal JSON reader for the dispatch table ---------------------------------------------------
struct Json {
  const char* p;
  const char* end;
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
  bool str(std::string& out) {
    ws();
    if (p >= end || *p != '"') return false;
    ++p;
    out.clear();
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) ++p;
      out.push_back(*p++);
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool num(long long& v) {
    ws();
    char* e = nullptr;
    v = strtoll(p, &e, 10);
    if (e == p) return false;
    p = e;
    return true;
  }
  bool skip_value() {
    ws();
    if (p >= end) return false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = (*p == '{') ? '}' : ']';
      int depth = 0;
      bool in_str = false;
      for (; p < end; ++p) {
        if (in_str) {
          if (*p == '\\') ++p;
          else if (*p == '"') in_str = false;
          continue;
        }
        if (*p == '"') in_str = true;
        else if (*p == open) ++depth;
        else if (*p == close && --depth == 0) {
          ++p;
          return true;
        }
      }
      return false;
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
};

int parse_family(const std::string& s) {
  if (s == "gemv") return S4_FAMILY_GEMV;
  if (s == "tc") return S4_FAMILY_TC;
  return -1;
}

bool parse_table(const char* text, std::vector<Bucket>& out, std::string& why) {
  Json j{text, text + strlen(text)};
  if (!j.lit('{')) return why = "expected '{'", false;
  bool found = false;
  while (true) {
    std::string key;
    if (j.lit('}')) break;
    if (!j.str(key) || !j.lit(':')) return why = "expected a key", false;
    if (key == "buckets") {
      found = true;
      if (!j.lit('[')) return why = "\"buckets\" must be an array", false;
      while (!j.lit(']')) {
        if (!j.lit('{')) return why = "bucket must be an object", false;
        Bucket b{INT_MAX, -1, 0, 0};
        while (!j.lit('}')) {
          std::string k;
          if (!j.str(k) || !j.lit(':')) return why = "bad bucket key", false;
          if (k == "family") {
            std::string f;
            if (!j.str(f) || (b.family = parse_family(f)) < 0) return why = "family must be \"gemv\" or \"tc\"", false;
          } else if (k == "fixup") {
            std::string f;
            if (!j.str(f)) return why = "fixup must be a string", false;
            if (f == "auto") b.fixup = s4::kFixupAuto;
            else if (f == "kernel") b.fixup = s4::kFixupKernel;
            else if (f == "cta") b.fixup = s4::kFixupCta;
            else return why = "fixup must be \"auto\", \"kernel\" or \"cta\"", false;
          } else if (k == "max_m" || k == "tile" || k == "split" || k == "K" || k == "N") {
            long long v;
            if (!j.num(v) || v < 0 || v > INT_MAX) return why = "bad number in bucket", false;
            (k == "max_m" ? b.max_m : k == "tile" ? b.tile : k == "split" ? b.split : k == "K" ? b.K : b.N) = (int)v;
          } else if (!j.skip_value()) {
            return why = "bad value", false;
          }
          j.lit(',');
        }
        if (b.family < 0) return why = "bucket without family", false;
        if (b.family == S4_FAMILY_TC && !s4::tc_available()) return why = "tc family is not built", false;
        if (b.family == S4_FAMILY_TC && b.tile != 0 && (b.tile < 16 || b.tile > 256 || b.tile % 16))
          return why = "tc tile must be 0 or a multiple of 16 in [16, 256]", false;
        // within one (K, N) key the buckets go up in M
        for (auto it = out.rbegin(); it != out.rend(); ++it)
          if (it->K == b.K && it->N == b.N) {
            if (b.max_m <= it->max_m) return why = "max_m must increase", false;
            break;
          }
        out.push_back(b);
        j.lit(',');
      }
    } else if (!j.skip_value()) {
      return why = "bad value", false;
    }
    j.lit(',');
  }
  if (!found || out.empty()) return why = "no buckets", false;
  // the last bucket for any shape covers every larger M; shape-specific buckets (K or N given) keep
  // their limit, and larger calls on those shapes fall through to the general buckets
  int last_any = -1;
  for (int i = 0; i < (int)out.size(); ++i)
    if (out[i].K == 0 && out[i].N == 0) last_any = i;
  if (last_any < 0) return why = "no bucket for every shape (one without K and N)", false;
  out[last_any].max_m = INT_MAX;
  return true;
}

int upload_common(s4_ctx* ctx, const void* packed_dev, const void* scales_dev, int N, int K, s4_weight** out,
                  const void* bias_dev = nullptr, int glu_I = 0) {
  s4_weight* w = new (std::nothrow) s4_weight();
  if (!w) return fail(S4_ERR_NOMEM, "out of host memory");
  w->ctx = ctx;
  w->device = ctx->device;
  w->sm_count = ctx->sm_count;
  w->N = N;
  w->K = K;
  w->glu = glu_I > 0;
  w->nblk = (N + s4::kRowsPerBlock - 1) / s4::kRowsPerBlock;
  w->ktiles = (K + s4::kKPerTile - 1) / s4::kKPerTile;
  w->wq_bytes = (size_t)w->nblk * w->ktiles * s4::kChunkWBytes;
  w->ws_bytes = (size_t)w->nblk * w->ktiles * s4::kChunkSBytes;
  cudaError_t e = cudaMalloc(&w->wq, w->wq_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->ws, w->ws_bytes);
  if (e == cudaSuccess && bias_dev) e = cudaMalloc(&w->wb, w->ws_bytes);
  if (e != cudaSuccess) {
    cudaFree(w->wq);
    cudaFree(w->ws);
    delete w;
    return fail(S4_ERR_NOMEM, "weight allocation of %zu bytes failed: %s", w->wq_bytes + w->ws_bytes,
                cudaGetErrorString(e));
  }
  e = s4::launch_repack(static_cast<const uint8_t*>(packed_dev), static_cast<const __half*>(scales_dev),
                        reinterpret_cast<uint32_t*>(w->wq), reinterpret_cast<__half*>(w->ws), N, K, w->nblk,
                        w->ktiles, ctx->sm_count, ctx->stream, glu_I);
  if (e == cudaSuccess && bias_dev) {
    ++ctx->launches;
    e = s4::launch_repack(nullptr, static_cast<const __half*>(bias_dev), nullptr, reinterpret_cast<__half*>(w->wb), N,
                          K, w->nblk, w->ktiles, ctx->sm_count, ctx->stream, 0);
  }
  if (e == cudaSuccess) {
    ++ctx->launches;
    e = cudaStreamSynchronize(ctx->stream);
  }
  if (e != cudaSuccess) {
    cudaFree(w->wq);
    cudaFree(w->ws);
    cudaFree(w->wb);
    delete w;
    return cuda_fail(e, "repack");
  }
  *out = w;
  return S4_OK;
}

int check_shape(int N, int K) {
  if (N < 1) return fail(S4_ERR_INVALID, "N must be >= 1 (got %d)", N);
  if (K < 32 || K % 32 != 0) return fail(S4_ERR_INVALID, "K must be a positive multiple of 32 (got %d)", K);
  const long long nblk = (N + 127) / 128;
  if (nblk > kMaxTickets) return fail(S4_ERR_INVALID, "N=%d exceeds the supported %d rows", N, kMaxTickets * 128);
  return S4_OK;
}

int grow(void** buf, size_t* cap, size_t need) {
  if (need <= *cap) return S4_OK;
  cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(buf, need);
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "staging allocation of %zu bytes failed", need);
  *cap = need;
  return S4_OK;
}

}  // namespace

extern "C" {

int s4_version(void) { return (1 << 16) | 0; }

const char* s4_last_error(void) { return g_last_error.c_str(); }

int s4_init(int device, s4_ctx** out) {
  if (!out) return fail(S4_ERR_INVALID, "out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(S4_ERR_UNSUPPORTED, "no CUDA device: %s", e != cudaSuccess ? cudaGetErrorString(e) : "count is 0");
  if (device < 0 || device >= count) return fail(S4_ERR_INVALID, "device %d out of range [0, %d)", device, count);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(S4_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                prop.minor);
  DeviceGuard guard(device);
  if (!guard.ok) return fail(S4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  s4_ctx* ctx = new (std::nothrow) s4_ctx();
  if (!ctx) return fail(S4_ERR_NOMEM, "out of host memory");
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  ctx->table = default_table();
  if (const char* v = getenv("S4_PDL")) ctx->pdl = (v[0] != '0');
  if (const char* v = getenv("S4_TICKET_FIXUP")) ctx->ticket_fixup = (v[0] == '1') ? 1 : 0;
  e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  const size_t part_bytes = s4::tc_partials_bytes(ctx->sm_count);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->partials, part_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->tickets, kMaxTickets * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->err, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->norm_ss, kNormSums * sizeof(float));
  if (e == cudaSuccess) e = cudaMemsetAsync(ctx->tickets, 0, kMaxTickets * sizeof(uint32_t), ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(ctx->err, 0, sizeof(uint32_t), ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    int rc = cuda_fail(e, "context allocation");
    s4_destroy(ctx);
    return rc;
  }
  *out = ctx;
  return S4_OK;
}

int s4_destroy(s4_ctx* ctx) {
  if (!ctx) return S4_OK;
  DeviceGuard guard(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->partials);
  cudaFree(ctx->tickets);
  cudaFree(ctx->err);
  cudaFree(ctx->norm_ss);
  cudaFree(ctx->dx);
  cudaFree(ctx->dy);
  cudaFree(ctx->wire_pow);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return S4_OK;
}

int s4_weight_upload(s4_ctx* ctx, const uint8_t* packed, const uint16_t* scales, int N, int K, uint32_t flags,
                     s4_weight** out) {
  if (!ctx || !packed || !scales || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (flags != 0) return fail(S4_ERR_INVALID, "unknown flags 0x%x", flags);
  int rc = check_shape(N, K);
  if (rc) return rc;
  DeviceGuard guard(ctx->device);
  const size_t pbytes = (size_t)N * (K / 32) * 16, sbytes = (size_t)N * (K / 32) * 2;
  void *dp = nullptr, *ds = nullptr;
  cudaError_t e = cudaMalloc(&dp, pbytes);
  if (e == cudaSuccess) e = cudaMalloc(&ds, sbytes);
  if (e != cudaSuccess) {
    cudaFree(dp);
    return fail(S4_ERR_NOMEM, "upload staging of %zu bytes failed", pbytes + sbytes);
  }
  e = cudaMemcpyAsync(dp, packed, pbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ds, scales, sbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(dp);
    cudaFree(ds);
    return cuda_fail(e, "upload copy");
  }
  rc = upload_common(ctx, dp, ds, N, K, out);
  cudaFree(dp);
  cudaFree(ds);
  return rc;
}

int s4_weight_upload_device(s4_ctx* ctx, const void* packed_dev, const void* scales_dev, int N, int K,
                            uint32_t flags, s4_weight** out) {
  if (!ctx || !packed_dev || !scales_dev || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (flags != 0) return fail(S4_ERR_INVALID, "unknown flags 0x%x", flags);
  if ((reinterpret_cast<uintptr_t>(packed_dev) & 3) || (reinterpret_cast<uintptr_t>(scales_dev) & 1))
    return fail(S4_ERR_INVALID, "packed must be 4-byte and scales 2-byte aligned");
  int rc = check_shape(N, K);
  if (rc) return rc;
  DeviceGuard guard(ctx->device);
  return upload_common(ctx, packed_dev, scales_dev, N, K, out);
}

// 2^(-r/4096), r in [0, 4096): libm pow returns the correctly rounded double for every one of them.
static int ensure_wire_table(s4_ctx* ctx) {
  if (ctx->wire_pow) return S4_OK;
  std::vector<double> t(4096);
  for (int r = 0; r < 4096; ++r) t[r] = std::pow(2.0, -r / 4096.0);
  double* d = nullptr;
  cudaError_t e = cudaMalloc(&d, t.size() * sizeof(double));
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "wire table allocation failed");
  e = cudaMemcpy(d, t.data(), t.size() * sizeof(double), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "wire table upload");
  }
  ctx->wire_pow = d;
  return S4_OK;
}

int s4_decode_wire_scales(s4_ctx* ctx, const void* wire_dev, int N, int G, void* scales_dev, void* stream) {
  if (!ctx || !wire_dev || !scales_dev) return fail(S4_ERR_INVALID, "NULL argument");
  if (N < 1 || G < 1) return fail(S4_ERR_INVALID, "bad shape N=%d G=%d", N, G);
  if (reinterpret_cast<uintptr_t>(scales_dev) & 1) return fail(S4_ERR_INVALID, "scales must be 2-byte aligned");
  DeviceGuard guard(ctx->device);
  int rc = ensure_wire_table(ctx);
  if (rc) return rc;
  cudaError_t e = s4::launch_wire_scales(static_cast<const uint8_t*>(wire_dev), N, G, ctx->wire_pow,
                                         static_cast<uint16_t*>(scales_dev), ctx->sm_count,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "wire scale decode launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_weight_upload_wire(s4_ctx* ctx, const uint8_t* packed, const uint8_t* wire_scales, int N, int K,
                          uint32_t flags, s4_weight** out) {
  if (!ctx || !packed || !wire_scales || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (flags != 0) return fail(S4_ERR_INVALID, "unknown flags 0x%x", flags);
  int rc = check_shape(N, K);
  if (rc) return rc;
  DeviceGuard guard(ctx->device);
  rc = ensure_wire_table(ctx);
  if (rc) return rc;
  const int G = K / 32;
  const size_t pbytes = (size_t)N * G * 16, sbytes = (size_t)N * G * 2, wbytes = 4 * (size_t)N + (size_t)N * G;
  uint8_t* d = nullptr;  // [packed | scales | wire]
  cudaError_t e = cudaMalloc(&d, pbytes + sbytes + wbytes);
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "upload staging of %zu bytes failed", pbytes + sbytes + wbytes);
  uint8_t *dp = d, *ds = d + pbytes, *dw = d + pbytes + sbytes;
  e = cudaMemcpyAsync(dp, packed, pbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dw, wire_scales, wbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) {
    e = s4::launch_wire_scales(dw, N, G, ctx->wire_pow, reinterpret_cast<uint16_t*>(ds), ctx->sm_count, ctx->stream);
    if (e == cudaSuccess) ++ctx->launches;
  }
  if (e != cudaSuccess) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    return cuda_fail(e, "wire upload");
  }
  rc = upload_common(ctx, dp, ds, N, K, out);  // same stream: runs after the decode
  cudaFree(d);
  return rc;
}

int s4_weight_upload_format(s4_ctx* ctx, const void* q, const void* scales, const void* bias, int N, int K, int bits,
                            int group, uint32_t flags, s4_weight** out) {
  if (!ctx || !q || !scales || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (flags & ~(S4_UPLOAD_DEVICE | S4_UPLOAD_DECODE_LAYOUT)) return fail(S4_ERR_INVALID, "unknown flags 0x%x", flags);
  if (bits < 2 || bits > 4) return fail(S4_ERR_INVALID, "bits must be 2, 3 or 4 (got %d)", bits);
  if ((flags & S4_UPLOAD_DECODE_LAYOUT) && (bits != 2 || bias))
    return fail(S4_ERR_UNSUPPORTED, "the native decode layout exists for symmetric 2-bit weights only");
  if (group != 32 && group != 64) return fail(S4_ERR_INVALID, "group must be 32 or 64 (got %d)", group);
  int rc = check_shape(N, K);
  if (rc) return rc;
  if (K % group) return fail(S4_ERR_INVALID, "K=%d is not a multiple of the group %d", K, group);
  const bool dev = flags & S4_UPLOAD_DEVICE;
  if (bits == 4 && group == 32 && !bias)
    return dev ? s4_weight_upload_device(ctx, q, scales, N, K, 0, out)
               : s4_weight_upload(ctx, static_cast<const uint8_t*>(q), static_cast<const uint16_t*>(scales), N, K, 0,
                                  out);
  if (dev && ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(scales) & 1) ||
              (reinterpret_cast<uintptr_t>(bias) & 1)))
    return fail(S4_ERR_INVALID, "q must be 4-byte and scales / bias 2-byte aligned");
  DeviceGuard guard(ctx->device);
  const size_t blocks = (size_t)N * (K / 32);
  const size_t qbytes = blocks * bits * 4, sbytes = (size_t)N * (K / group) * 2;
  const size_t p4 = blocks * 16, s32 = blocks * 2, b32 = bias ? s32 : 0;
  const size_t in_bytes = dev ? 0 : qbytes + sbytes + (bias ? sbytes : 0);
  const size_t total = p4 + s32 + b32 + in_bytes;
  uint8_t* d = nullptr;  // [packed int4 | scales per 32 | biases per 32 | (host input: q | scales | bias)]
  cudaError_t e = cudaMalloc(&d, total);
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "format staging of %zu bytes failed", total);
  __half* ds32 = reinterpret_cast<__half*>(d + p4);
  __half* db32 = bias ? reinterpret_cast<__half*>(d + p4 + s32) : nullptr;
  const void *dq = q, *dsc = scales, *dbi = bias;
  if (!dev) {
    uint8_t* in = d + p4 + s32 + b32;
    dq = in;
    dsc = in + qbytes;
    dbi = bias ? in + qbytes + sbytes : nullptr;
    e = cudaMemcpyAsync(const_cast<void*>(dq), q, qbytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(const_cast<void*>(dsc), scales, sbytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && bias)
      e = cudaMemcpyAsync(const_cast<void*>(dbi), bias, sbytes, cudaMemcpyHostToDevice, ctx->stream);
  }
  if (e == cudaSuccess) {
    e = s4::launch_transcode(static_cast<const uint32_t*>(dq), static_cast<const __half*>(dsc),
                             static_cast<const __half*>(dbi), N, K, bits, group, d, ds32, db32, ctx->sm_count,
                             ctx->stream);
    if (e == cudaSuccess) ++ctx->launches;
  }
  if (e != cudaSuccess) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    return cuda_fail(e, "format upload");
  }
  rc = upload_common(ctx, d, ds32, N, K, out, db32);
  if (rc == S4_OK && (flags & S4_UPLOAD_DECODE_LAYOUT)) {
    // symmetric 2-bit: also the native 2-bit decode layout, which the decode GEMV streams (2048 weight
    // bytes per chunk instead of 4096); the int4 layout stays for the tcgen05 GEMM and chained runs
    s4_weight* w = *out;
    w->wq2_bytes = (size_t)w->nblk * w->ktiles * 2048;
    e = cudaMalloc(&w->wq2, w->wq2_bytes);
    if (e == cudaSuccess) {
      e = s4::launch_repack2(static_cast<const uint32_t*>(dq), N, K, w->nblk, w->ktiles, w->wq2, ctx->sm_count,
                             ctx->stream);
      if (e == cudaSuccess) ++ctx->launches;
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(d);
      s4_weight_free(w);
      *out = nullptr;
      return cuda_fail(e, "2-bit decode layout");
    }
  }
  cudaFree(d);
  return rc;
}

int s4_fwht(s4_ctx* ctx, void* a, int M, int K, int n, void* stream) {
  if (!ctx || !a) return fail(S4_ERR_INVALID, "NULL argument");
  if (M < 0 || K < 1) return fail(S4_ERR_INVALID, "bad shape M=%d K=%d", M, K);
  if (n < 2 || n > 32768 || (n & (n - 1))) return fail(S4_ERR_INVALID, "n must be a power of two in [2, 32768] (got %d)", n);
  if (K % n) return fail(S4_ERR_INVALID, "K=%d is not a multiple of n=%d", K, n);
  if (reinterpret_cast<uintptr_t>(a) & 1) return fail(S4_ERR_INVALID, "a must be 2-byte aligned");
  if (M == 0) return S4_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_fwht(static_cast<__half*>(a), (int64_t)M * (K / n), n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fwht launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_weight_upload_glu(s4_ctx* ctx, const void* packed, const void* scales, int I, int K, uint32_t flags,
                         s4_weight** out) {
  if (!ctx || !packed || !scales || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (flags & ~S4_UPLOAD_DEVICE) return fail(S4_ERR_INVALID, "unknown flags 0x%x", flags);
  if (I < 64 || I % 64) return fail(S4_ERR_INVALID, "I must be a positive multiple of 64 (got %d)", I);
  int rc = check_shape(2 * I, K);
  if (rc) return rc;
  DeviceGuard guard(ctx->device);
  if (flags & S4_UPLOAD_DEVICE) {
    if ((reinterpret_cast<uintptr_t>(packed) & 3) || (reinterpret_cast<uintptr_t>(scales) & 1))
      return fail(S4_ERR_INVALID, "packed must be 4-byte and scales 2-byte aligned");
    return upload_common(ctx, packed, scales, 2 * I, K, out, nullptr, I);
  }
  const size_t pbytes = (size_t)2 * I * (K / 32) * 16, sbytes = (size_t)2 * I * (K / 32) * 2;
  uint8_t* d = nullptr;
  cudaError_t e = cudaMalloc(&d, pbytes + sbytes);
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "upload staging of %zu bytes failed", pbytes + sbytes);
  e = cudaMemcpyAsync(d, packed, pbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d + pbytes, scales, sbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    return cuda_fail(e, "upload copy");
  }
  rc = upload_common(ctx, d, d + pbytes, 2 * I, K, out, nullptr, I);
  cudaFree(d);
  return rc;
}

int s4_weight_free(s4_weight* w) {
  if (!w) return S4_OK;
  DeviceGuard guard(w->device);
  cudaFree(w->wq);
  cudaFree(w->ws);
  cudaFree(w->wb);
  cudaFree(w->wq2);
  delete w;
  return S4_OK;
}

int s4_weight_info(const s4_weight* w, int* N, int* K, size_t* device_bytes) {
  if (!w) return fail(S4_ERR_INVALID, "NULL weight");
  if (N) *N = w->N;
  if (K) *K = w->K;
  if (device_bytes) *device_bytes = w->wq_bytes + w->ws_bytes + (w->wb ? w->ws_bytes : 0) + w->wq2_bytes;
  if (N && w->glu) *N = w->N / 2;  // a fused gate|up weight's matmul writes N / 2 columns
  return S4_OK;
}

int s4_weight_layout_bytes(const s4_weight* w, size_t* wq_bytes, size_t* ws_bytes) {
  if (!w) return fail(S4_ERR_INVALID, "NULL weight");
  if (wq_bytes) *wq_bytes = w->wq_bytes;
  if (ws_bytes) *ws_bytes = w->ws_bytes;
  return S4_OK;
}

int s4_weight_download_layout(const s4_weight* w, void* wq_host, size_t wq_bytes, void* ws_host, size_t ws_bytes) {
  if (!w || !wq_host || !ws_host) return fail(S4_ERR_INVALID, "NULL argument");
  if (wq_bytes < w->wq_bytes || ws_bytes < w->ws_bytes) return fail(S4_ERR_INVALID, "host buffers too small");
  DeviceGuard guard(w->device);
  cudaError_t e = cudaMemcpy(wq_host, w->wq, w->wq_bytes, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(ws_host, w->ws, w->ws_bytes, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "layout download");
  return S4_OK;
}

// ---- on-disk cache of repacked weights ----
namespace {
constexpr uint32_t kCacheMagic = 0x4c573453u;  // "S4WL"
constexpr uint32_t kCacheLayoutVersion = 1;    // the device layout of repack.cu; bump when it changes
struct CacheHeader {
  uint32_t magic, version;
  int32_t N, K;
  uint32_t flags;  // bit 0: asymmetric (a bias section follows the scales); bit 1: fused gate|up (SiLU*mul)
  uint32_t reserved0;
  uint64_t wq_bytes, ws_bytes, wb_bytes;
  uint64_t checksum;  // of the payload, cache_checksum()
  uint64_t reserved1;
};
static_assert(sizeof(CacheHeader) == 64, "cache header is 64 bytes");

// FNV-1a style over 8-byte little-endian words with an extra xor-shift per word (multi-byte words
// need the high bits folded back); detects truncation and corruption, not tampering.
uint64_t cache_checksum(const uint8_t* p, size_t n, uint64_t h) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    memcpy(&w, p + i, 8);
    h = (h ^ w) * 0x100000001b3ull;
    h ^= h >> 29;
  }
  uint64_t w = 0;
  memcpy(&w, p + i, n - i);
  h = (h ^ w ^ (uint64_t)n) * 0x100000001b3ull;
  return h ^ (h >> 29);
}
}  // namespace

int s4_weight_save(const s4_weight* w, const char* path) {
  if (!w || !path) return fail(S4_ERR_INVALID, "NULL argument");
  const size_t wb_bytes = w->wb ? w->ws_bytes : 0;
  std::vector<uint8_t> buf;
  try {
    buf.resize(w->wq_bytes + w->ws_bytes + wb_bytes);
  } catch (const std::bad_alloc&) {
    return fail(S4_ERR_NOMEM, "out of host memory for the cache copy");
  }
  {
    DeviceGuard guard(w->device);
    cudaError_t e = cudaMemcpy(buf.data(), w->wq, w->wq_bytes, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(buf.data() + w->wq_bytes, w->ws, w->ws_bytes, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && w->wb)
      e = cudaMemcpy(buf.data() + w->wq_bytes + w->ws_bytes, w->wb, wb_bytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "weight download for the cache");
  }
  CacheHeader h = {};
  h.magic = kCacheMagic;
  h.version = kCacheLayoutVersion;
  h.N = w->N;
  h.K = w->K;
  h.flags = (w->wb ? 1u : 0u) | (w->glu ? 2u : 0u);
  h.wq_bytes = w->wq_bytes;
  h.ws_bytes = w->ws_bytes;
  h.wb_bytes = wb_bytes;
  h.checksum = cache_checksum(buf.data(), buf.size(), 0xcbf29ce484222325ull);
  const std::string tmp = std::string(path) + ".tmp";  // written whole, then renamed over the entry
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return fail(S4_ERR_IO, "cannot create %s", tmp.c_str());
  const bool ok = fwrite(&h, sizeof h, 1, f) == 1 && fwrite(buf.data(), 1, buf.size(), f) == buf.size();
  const bool closed = fclose(f) == 0;
  if (!ok || !closed || rename(tmp.c_str(), path) != 0) {
    remove(tmp.c_str());
    return fail(S4_ERR_IO, "writing %s failed", path);
  }
  return S4_OK;
}

int s4_weight_load(s4_ctx* ctx, const char* path, s4_weight** out) {
  if (!ctx || !path || !out) return fail(S4_ERR_INVALID, "NULL argument");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(S4_ERR_IO, "no cache entry %s", path);
  CacheHeader h;
  if (fread(&h, sizeof h, 1, f) != 1) {
    fclose(f);
    return fail(S4_ERR_IO, "%s: truncated header", path);
  }
  if (h.magic != kCacheMagic || h.version != kCacheLayoutVersion || (h.flags & ~3u)) {
    fclose(f);
    return fail(S4_ERR_IO, "%s: not a weight of layout version %u", path, kCacheLayoutVersion);
  }
  if (check_shape(h.N, h.K) != S4_OK) {
    fclose(f);
    return fail(S4_ERR_IO, "%s: bad shape N=%d K=%d", path, h.N, h.K);
  }
  s4_weight* w = new (std::nothrow) s4_weight();
  if (!w) {
    fclose(f);
    return fail(S4_ERR_NOMEM, "out of host memory");
  }
  w->ctx = ctx;
  w->device = ctx->device;
  w->sm_count = ctx->sm_count;
  w->N = h.N;
  w->K = h.K;
  w->glu = (h.flags & 2u) ? 1 : 0;
  w->nblk = (h.N + s4::kRowsPerBlock - 1) / s4::kRowsPerBlock;
  w->ktiles = (h.K + s4::kKPerTile - 1) / s4::kKPerTile;
  w->wq_bytes = (size_t)w->nblk * w->ktiles * s4::kChunkWBytes;
  w->ws_bytes = (size_t)w->nblk * w->ktiles * s4::kChunkSBytes;
  const size_t wb_bytes = (h.flags & 1u) ? w->ws_bytes : 0;
  if (h.wq_bytes != w->wq_bytes || h.ws_bytes != w->ws_bytes || h.wb_bytes != wb_bytes) {
    fclose(f);
    delete w;
    return fail(S4_ERR_IO, "%s: section sizes do not match N=%d K=%d", path, h.N, h.K);
  }
  // the payload must be exactly the rest of the file: checked before any buffer is sized from the
  // header, so a damaged or foreign header cannot ask for an arbitrary allocation
  const size_t payload = w->wq_bytes + w->ws_bytes + wb_bytes;
  const off_t here = ftello(f);
  const bool sized = here >= 0 && fseeko(f, 0, SEEK_END) == 0 && ftello(f) - here == (off_t)payload &&
                     fseeko(f, here, SEEK_SET) == 0;
  if (!sized) {
    fclose(f);
    delete w;
    return fail(S4_ERR_IO, "%s: truncated or corrupt payload", path);
  }
  std::vector<uint8_t> buf;
  try {
    buf.resize(payload);
  } catch (const std::bad_alloc&) {
    fclose(f);
    delete w;
    return fail(S4_ERR_NOMEM, "out of host memory for %s", path);
  }
  const bool read_ok = fread(buf.data(), 1, buf.size(), f) == buf.size() && fgetc(f) == EOF;
  fclose(f);
  if (!read_ok || cache_checksum(buf.data(), buf.size(), 0xcbf29ce484222325ull) != h.checksum) {
    delete w;
    return fail(S4_ERR_IO, "%s: truncated or corrupt payload", path);
  }
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMalloc(&w->wq, w->wq_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->ws, w->ws_bytes);
  if (e == cudaSuccess && wb_bytes) e = cudaMalloc(&w->wb, wb_bytes);
  if (e == cudaSuccess) e = cudaMemcpy(w->wq, buf.data(), w->wq_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(w->ws, buf.data() + w->wq_bytes, w->ws_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && wb_bytes)
    e = cudaMemcpy(w->wb, buf.data() + w->wq_bytes + w->ws_bytes, wb_bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(w->wq);
    cudaFree(w->ws);
    cudaFree(w->wb);
    delete w;
    return cuda_fail(e, "cache load");
  }
  *out = w;
  return S4_OK;
}

// Tokens per tcgen05 tile when the table does not fix it: 256 (M rounded up to 16 below that);
// 128 when K is short (<= 4096) and 256-token tiles would fill under 3/4 of the SMs while 128-token
// tiles still fit in one wave (measured: out_proj M = 256..1024, in_proj M = 256 faster by 20-25%;
// long-K shapes keep 256, their split tiles are cheap relative to the main loop).
static int auto_tile(int M, const s4_weight* w, int sms) {
  if (M < 256) return ((M + 15) / 16) * 16;
  const long long t256 = (long long)((M + 255) / 256) * w->nblk, t128 = (long long)((M + 127) / 128) * w->nblk;
  if (w->K <= 4096 && t256 * 4 < (long long)sms * 3 && t128 <= sms) return 128;
  return 256;
}

// Split tiles of a launch summed by their last CTA (in-kernel) or by the fix-up kernel: the table's
// choice, else the environment's (S4_TICKET_FIXUP), else the fix-up kernel. The tuner measured the
// in-kernel form slower on every shape and M of the sweep (1.2x with two parts per tile, up to 6x with
// ten): one CTA's four epilogue warps sum the other parts 16 rows at a time, a chain of L2 round
// trips, while the fix-up kernel spreads the same reads over the whole grid. Fused gate|up weights
// always use the fix-up kernel (it pairs gate and up rows).
static bool use_cta_fixup(const Bucket& b, const s4_ctx* ctx, const s4_weight* w) {
  if (w->glu) return false;
  if (b.fixup == s4::kFixupCta) return true;
  if (b.fixup == s4::kFixupKernel) return false;
  return ctx->ticket_fixup == 1;
}

// Tile size and CTA count together. Two cases where whole tiles packed into whole waves beat the
// default split (measured on gate|up, down, out_proj): (1) 256-token tiles fit in one wave: as many
// token blocks as fit, if their tiles stay >= 224 tokens (down / out_proj M = 2048: 144 tiles of 240
// instead of 128 of 256, +3 %); (2) they need one to two waves: two exact waves of whole tiles of >= 176
// tokens when those keep >= 95 % of the SMs busy (gate|up M = 512: 288 tiles of 176 on 144 CTAs, no
// split tiles and no fix-up, +11 %).
static void auto_shape(int M, const s4_weight* w, int sms, int* tn_out, int* grid_out) {
  int tn = auto_tile(M, w, sms), grid = sms;
  const long long nb = w->nblk, t256 = (long long)((M + 255) / 256) * nb;
  if (tn == 256 && t256 <= sms) {
    const long long b = sms / nb;  // token blocks that fit one wave
    if (b > 0) {
      const int t = (int)((((long long)M + b - 1) / b + 15) / 16 * 16);
      if (t >= 224 && t < 256) tn = t;
    }
  } else if (tn == 256 && t256 <= 2LL * sms) {
    const long long b = 2LL * sms / nb;  // token blocks that fit two waves
    if (b > 0) {
      const int t = (int)((((long long)M + b - 1) / b + 15) / 16 * 16);
      const long long tiles = (long long)((M + t - 1) / t) * nb;
      if (t >= 176 && t <= 256 && tiles % 2 == 0 && (tiles / 2) * 100 >= (long long)sms * 95) {
        tn = t;
        grid = (int)(tiles / 2);
      }
    }
  }
  // fewer tiles than CTAs but at least 60 % as many: one whole tile per CTA (the idle SMs cost less
  // than splitting every tile and fixing it up: gate|up at M = 64..256, 96 tiles for 148 SMs, ran
  // 7-22 % faster whole; at 65 tiles for 148 SMs splitting still won)
  const long long tiles = (long long)((M + tn - 1) / tn) * nb;
  if (tiles < grid && tiles * 5 >= (long long)grid * 3) grid = (int)tiles;
  // more tiles than CTAs: whole waves of whole tiles when a CTA count of at least 85 % of the SMs
  // divides the tile count (no split tile, no fix-up launch) and costs each CTA at most one tile more
  // than stream-K over every SM would; measured against stream-K: gate|up M = 1024 / 2048 on 128
  // CTAs 16 / 7.5 % faster, the fused qkvz|ab projection on 130 CTAs 26 / 12 % faster; at many waves
  // (8192-token serving chunks) the idle SMs cost more than the split tiles
  if (tiles > grid && grid == sms)
    for (long long g = sms; g * 100 >= (long long)sms * 85; --g)
      if (tiles % g == 0) {
        if (tiles * (sms - g) <= g * (long long)sms) grid = (int)g;
        break;
      }
  *tn_out = tn;
  *grid_out = grid;
}

// Tokens per tile, CTAs and fix-up form of a tcgen05 launch for bucket b (the table's values, the
// automatic shape where it gives 0). s4_matmul and s4_matmul_gather both use it, so the two entry
// points split a matmul's K range the same way and agree bit for bit.
static int tc_launch_shape(const s4_ctx* ctx, const s4_weight* w, const Bucket& b, int M, int* tn, int* grid,
                           bool* cta_fixup) {
  const bool tc = b.family == S4_FAMILY_TC;
  if (tc && b.tile != 0 && (b.tile < 16 || b.tile > 256 || b.tile % 16))
    return fail(S4_ERR_INVALID, "tc tile must be a multiple of 16 in [16, 256] (got %d)", b.tile);
  *tn = tc ? b.tile : 0;
  *grid = ctx->sm_count;
  if (*tn == 0) auto_shape(M, w, ctx->sm_count, tn, grid);
  if (tc && b.split > 0) *grid = std::min(b.split, ctx->sm_count);
  *cta_fixup = tc && use_cta_fixup(b, ctx, w);
  return S4_OK;
}

int s4_matmul(s4_ctx* ctx, const s4_weight* w, const void* x, int M, void* y, void* stream) {
  if (!ctx || !w) return fail(S4_ERR_INVALID, "NULL context or weight");
  if (w->ctx != ctx) return fail(S4_ERR_INVALID, "weight belongs to another context");
  if (M < 0) return fail(S4_ERR_INVALID, "M must be >= 0 (got %d)", M);
  if (M == 0) return S4_OK;
  if (!x || !y) return fail(S4_ERR_INVALID, "NULL x or y");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return fail(S4_ERR_INVALID, "x and y must be 16-byte aligned");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Bucket b = choose(ctx, M, w->N, w->K);
  cudaError_t e = cudaSuccess;
  if (b.family == S4_FAMILY_TC) {
    int tn = 0, grid = 0;
    bool cta = false;
    const int rc = tc_launch_shape(ctx, w, b, M, &tn, &grid, &cta);
    if (rc != S4_OK) return rc;
    // token rows per launch: the arrival counters hold one entry per (token block, n-block) tile
    const long long rows_cap = (long long)(kMaxTickets / w->nblk) * tn;
    for (long long r0 = 0; r0 < M; r0 += rows_cap) {
      const int rows = (int)std::min<long long>(rows_cap, M - r0);
      e = s4::launch_tc_gemm(w->wq, w->ws, w->wb, static_cast<const __half*>(x) + r0 * w->K,
                             static_cast<__half*>(y) + r0 * (w->glu ? w->N / 2 : w->N), ctx->partials, ctx->tickets,
                             kMaxTickets, ctx->err, rows, w->N, w->K, w->nblk, w->ktiles, tn, grid, st, ctx->pdl,
                             cta, w->glu);
      if (e != cudaSuccess) return cuda_fail(e, "tc gemm launch");
      ++ctx->launches;
    }
    return S4_OK;
  }
  for (int tok0 = 0; tok0 < M; tok0 += kGemvMaxM) {
    const int rem = M - tok0;
    const int groups = rem >= kGemvMaxM ? kGemvMaxM / 8 : (rem + 7) / 8;
    e = s4::launch_gemv(w->wq, w->ws, w->wb, static_cast<const __half*>(x), static_cast<__half*>(y), ctx->err, M, w->N,
                        w->K, w->nblk, w->ktiles, tok0, groups, b.split, ctx->sm_count, st, ctx->pdl, w->glu,
                        w->wq2);
    if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    ++ctx->launches;
  }
  return S4_OK;
}

int s4_matmul_host(s4_ctx* ctx, const s4_weight* w, const uint16_t* x, int M, uint16_t* y) {
  if (!ctx || !w) return fail(S4_ERR_INVALID, "NULL context or weight");
  if (M < 0) return fail(S4_ERR_INVALID, "M must be >= 0 (got %d)", M);
  if (M == 0) return S4_OK;
  if (!x || !y) return fail(S4_ERR_INVALID, "NULL x or y");
  DeviceGuard guard(ctx->device);
  const size_t xb = (size_t)M * w->K * 2, yb = (size_t)M * (w->glu ? w->N / 2 : w->N) * 2;
  if (xb > ctx->dx_cap || yb > ctx->dy_cap) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "staging resize");
  }
  int rc = grow(&ctx->dx, &ctx->dx_cap, xb);
  if (!rc) rc = grow(&ctx->dy, &ctx->dy_cap, yb);
  if (rc) return rc;
  cudaError_t e = cudaMemcpyAsync(ctx->dx, x, xb, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "x upload");
  rc = s4_matmul(ctx, w, ctx->dx, M, ctx->dy, ctx->stream);
  if (rc) return rc;
  e = cudaMemcpyAsync(y, ctx->dy, yb, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "y download");
  return S4_OK;
}

int s4_matmul_host_async(s4_ctx* ctx, const s4_weight* w, const uint16_t* x, int M, uint16_t* y, void* stream) {
  if (!ctx || !w) return fail(S4_ERR_INVALID, "NULL context or weight");
  if (M < 0) return fail(S4_ERR_INVALID, "M must be >= 0 (got %d)", M);
  if (M == 0) return S4_OK;
  if (!x || !y) return fail(S4_ERR_INVALID, "NULL x or y");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t xb = (size_t)M * w->K * 2, yb = (size_t)M * (w->glu ? w->N / 2 : w->N) * 2;
  if (xb > ctx->dx_cap || yb > ctx->dy_cap) {
    // growing frees the old staging buffers: wait for work that may still use them
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "staging resize");
  }
  int rc = grow(&ctx->dx, &ctx->dx_cap, xb);
  if (!rc) rc = grow(&ctx->dy, &ctx->dy_cap, yb);
  if (rc) return rc;
  cudaError_t e = cudaMemcpyAsync(ctx->dx, x, xb, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "x upload");
  rc = s4_matmul(ctx, w, ctx->dx, M, ctx->dy, stream);
  if (rc) return rc;
  e = cudaMemcpyAsync(y, ctx->dy, yb, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "y download");
  return S4_OK;
}

int s4_silu_mul(s4_ctx* ctx, const void* big, int M, int I, void* mid, void* stream) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  if (M < 0 || I < 1) return fail(S4_ERR_INVALID, "bad shape M=%d I=%d", M, I);
  if (M == 0) return S4_OK;
  if (!big || !mid) return fail(S4_ERR_INVALID, "NULL big or mid");
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_silu_mul(static_cast<const __half*>(big), static_cast<__half*>(mid), M, I, ctx->sm_count,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "silu_mul launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_chain_create(s4_ctx* ctx, int nops, const s4_weight* const* w, const void* const* x, void* const* y,
                    const int* M, const int* dep, s4_chain** out) {
  if (!ctx || !w || !x || !y || !M || !out) return fail(S4_ERR_INVALID, "NULL argument");
  if (nops < 1) return fail(S4_ERR_INVALID, "nops must be >= 1 (got %d)", nops);
  for (int i = 0; i < nops; ++i) {
    if (!w[i] || !x[i] || !y[i]) return fail(S4_ERR_INVALID, "NULL weight or buffer in op %d", i);
    if (w[i]->ctx != ctx) return fail(S4_ERR_INVALID, "op %d: weight belongs to another context", i);
  }
  DeviceGuard guard(ctx->device);
  const char* why = nullptr;
  int rc;
  try {  // host containers sized by nops: an allocation failure is a status, not an exception
    rc = s4::chain_create(ctx, nops, w, x, y, M, dep, out, &why);
  } catch (const std::bad_alloc&) {
    return fail(S4_ERR_NOMEM, "chain: out of host memory");
  }
  if (rc != S4_OK) return fail(rc, "chain: %s", why ? why : "failed");
  return S4_OK;
}

int s4_chain_run(s4_ctx* ctx, s4_chain* chain, void* stream) {
  if (!ctx || !chain) return fail(S4_ERR_INVALID, "NULL argument");
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::chain_launch(chain, ctx->err, static_cast<cudaStream_t>(stream), !ctx->pdl);
  if (e != cudaSuccess) return cuda_fail(e, "chain launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_chain_run_host(s4_ctx* ctx, s4_chain* chain, const void* x_host, void* x_dev, size_t x_bytes, void* y_host,
                      const void* y_dev, size_t y_bytes, void* stream) {
  if (!ctx || !chain) return fail(S4_ERR_INVALID, "NULL argument");
  if ((x_bytes && (!x_host || !x_dev)) || (y_bytes && (!y_host || !y_dev)))
    return fail(S4_ERR_INVALID, "NULL host or device buffer");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = x_bytes ? cudaMemcpyAsync(x_dev, x_host, x_bytes, cudaMemcpyHostToDevice, st) : cudaSuccess;
  if (e != cudaSuccess) return cuda_fail(e, "chain input upload");
  e = s4::chain_launch(chain, ctx->err, st, true);  // callers alternate streams between host-buffer runs
  if (e != cudaSuccess) return cuda_fail(e, "chain launch");
  ++ctx->launches;
  e = y_bytes ? cudaMemcpyAsync(y_host, y_dev, y_bytes, cudaMemcpyDeviceToHost, st) : cudaSuccess;
  if (e != cudaSuccess) return cuda_fail(e, "chain output download");
  return S4_OK;
}

int s4_chain_info(const s4_chain* chain, int* grid, int* slots, int* smem_bytes) {
  if (!chain) return fail(S4_ERR_INVALID, "NULL chain");
  return s4::chain_info(chain, grid, slots, smem_bytes);
}

int s4_chain_free(s4_chain* chain) {
  if (!chain) return S4_OK;
  s4::chain_destroy(chain);
  return S4_OK;
}

static int add_rmsnorm_impl(s4_ctx* ctx, float* x, const void* y, const float* w, int M, int D, float eps, void* h,
                            const void* own_flags, int nranks, void* stream) {
  if (!ctx || !x || !h) return fail(S4_ERR_INVALID, "NULL argument");
  if (M < 0 || D < 1) return fail(S4_ERR_INVALID, "bad shape M=%d D=%d", M, D);
  if (own_flags && (nranks < 1 || nranks > 8)) return fail(S4_ERR_INVALID, "nranks must be in [1, 8]");
  if (M == 0) return S4_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_add_rmsnorm(x, static_cast<const __half*>(y), w, M, D, eps, static_cast<__half*>(h),
                                         static_cast<cudaStream_t>(stream), static_cast<const uint32_t*>(own_flags),
                                         nranks, ctx->err);
  if (e != cudaSuccess) return cuda_fail(e, "add_rmsnorm launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_add_rmsnorm(s4_ctx* ctx, float* x, const void* y, const float* w, int M, int D, float eps, void* h,
                   void* stream) {
  return add_rmsnorm_impl(ctx, x, y, w, M, D, eps, h, nullptr, 0, stream);
}

int s4_add_rmsnorm_wait(s4_ctx* ctx, float* x, const void* y, const float* w, int M, int D, float eps, void* h,
                        const void* own_flags, int nranks, void* stream) {
  if (!own_flags) return fail(S4_ERR_INVALID, "NULL flag array");
  return add_rmsnorm_impl(ctx, x, y, w, M, D, eps, h, own_flags, nranks, stream);
}

int s4_matmul_add_rmsnorm(s4_ctx* ctx, const s4_weight* w, const void* x, int M, float* resid, const float* norm_w,
                          float eps, void* h, void* stream) {
  if (!ctx || !w) return fail(S4_ERR_INVALID, "NULL context or weight");
  if (w->ctx != ctx) return fail(S4_ERR_INVALID, "weight belongs to another context");
  if (M < 0) return fail(S4_ERR_INVALID, "M must be >= 0 (got %d)", M);
  if (M == 0) return S4_OK;
  if (!x || !resid || !h) return fail(S4_ERR_INVALID, "NULL x, residual or h");
  if (w->glu) return fail(S4_ERR_UNSUPPORTED, "a fused gate|up weight has no residual epilogue");
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(x) || misaligned(resid) || misaligned(h) || (norm_w && misaligned(norm_w)))
    return fail(S4_ERR_INVALID, "x, residual, norm weight and h must be 16-byte aligned");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int N = w->N;
  const Bucket b = choose(ctx, M, N, w->K);
  if (b.family == S4_FAMILY_TC && N % 32 == 0) {
    // the residual add and the per-32-column sums of squares in the GEMM epilogue, then one row pass
    int tn = 0, grid = 0;
    bool cta = false;
    const int rc = tc_launch_shape(ctx, w, b, M, &tn, &grid, &cta);
    if (rc != S4_OK) return rc;
    const long long rows_cap = std::min<long long>((long long)(kMaxTickets / w->nblk) * tn,
                                                   (long long)(kNormSums / (size_t)(N / 32)));
    for (long long r0 = 0; r0 < M; r0 += rows_cap) {
      const int rows = (int)std::min<long long>(rows_cap, M - r0);
      __half* hr = static_cast<__half*>(h) + r0 * N;
      float* xr = resid + r0 * N;
      cudaError_t e = s4::launch_tc_gemm_ex(w->wq, w->ws, w->wb, static_cast<const __half*>(x) + r0 * w->K, w->K, &hr,
                                            1, N, 0, ctx->partials, ctx->tickets, kMaxTickets, ctx->err, rows, N, w->K,
                                            w->nblk, w->ktiles, tn, grid, st, ctx->pdl, false, 0, xr, N, ctx->norm_ss,
                                            rows, nullptr, 0);
      if (e != cudaSuccess) return cuda_fail(e, "tc gemm launch (residual epilogue)");
      e = s4::launch_rmsnorm_from_sums(xr, ctx->norm_ss, rows, norm_w, rows, N, eps, hr, st, ctx->pdl);
      if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
      ctx->launches += 2;
    }
    return S4_OK;
  }
  // other families: y into h, then ADD_NORM over it in place
  int rc = s4_matmul(ctx, w, x, M, h, stream);
  if (rc != S4_OK) return rc;
  cudaError_t e = s4::launch_add_rmsnorm(resid, static_cast<const __half*>(h), norm_w, M, N, eps,
                                         static_cast<__half*>(h), st, nullptr, 0, nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "add_rmsnorm launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_buffer_alloc(s4_ctx* ctx, size_t bytes, void** ptr) {
  if (!ctx || !ptr || bytes == 0) return fail(S4_ERR_INVALID, "bad argument");
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return fail(S4_ERR_NOMEM, "buffer allocation of %zu bytes failed", bytes);
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "buffer clear");
  return S4_OK;
}

int s4_buffer_free(s4_ctx* ctx, void* ptr) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "buffer free");
  return S4_OK;
}

int s4_ipc_handle(s4_ctx* ctx, const void* ptr, void* handle64) {
  if (!ctx || !ptr || !handle64) return fail(S4_ERR_INVALID, "NULL argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  DeviceGuard guard(ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle64, &h, sizeof(h));
  return S4_OK;
}

int s4_ipc_open(s4_ctx* ctx, const void* handle64, void** ptr) {
  if (!ctx || !handle64 || !ptr) return fail(S4_ERR_INVALID, "NULL argument");
  DeviceGuard guard(ctx->device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return S4_OK;
}

int s4_ipc_close(s4_ctx* ctx, void* ptr) {
  if (!ctx || !ptr) return fail(S4_ERR_INVALID, "NULL argument");
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return S4_OK;
}

static int matmul_gather_impl(s4_ctx* ctx, const s4_weight* w, const void* x, int ldx, int M, void* const* dst,
                              int ndst, int ldy, int col0, const void* own_flags, int nranks, void* stream) {
  if (!ctx || !w || !dst) return fail(S4_ERR_INVALID, "NULL argument");
  if (own_flags && (nranks < 1 || nranks > 8)) return fail(S4_ERR_INVALID, "nranks must be in [1, 8]");
  if (w->ctx != ctx) return fail(S4_ERR_INVALID, "weight belongs to another context");
  if (M < 0 || ndst < 1 || ndst > 8) return fail(S4_ERR_INVALID, "bad M or ndst");
  if (M == 0) return S4_OK;
  if (!x || ldx < w->K || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(S4_ERR_INVALID, "x must be 16-byte aligned with ldx >= K and ldx*2 a multiple of 16");
  const int ycols = w->glu ? w->N / 2 : w->N;
  if (ldy < 1 || col0 < 0 || (long long)col0 + ycols > ldy) return fail(S4_ERR_INVALID, "output slice outside the row");
  for (int d = 0; d < ndst; ++d)
    if (!dst[d]) return fail(S4_ERR_INVALID, "NULL destination %d", d);
  DeviceGuard guard(ctx->device);
  // the dispatch table's tcgen05 shape for this weight and M (a GEMV bucket: the automatic shape), the
  // same split as s4_matmul's
  int tn = 0, grid = 0;
  bool cta = false;
  const int rc = tc_launch_shape(ctx, w, choose(ctx, M, w->N, w->K), M, &tn, &grid, &cta);
  if (rc != S4_OK) return rc;
  if ((long long)((M + tn - 1) / tn) * w->nblk > kMaxTickets) return fail(S4_ERR_INVALID, "M too large for one launch");
  cudaError_t e = s4::launch_tc_gemm_ex(w->wq, w->ws, w->wb, static_cast<const __half*>(x), ldx,
                                        reinterpret_cast<__half* const*>(dst), ndst, ldy, col0, ctx->partials,
                                        ctx->tickets, kMaxTickets, ctx->err, M, w->N, w->K, w->nblk, w->ktiles, tn,
                                        grid, static_cast<cudaStream_t>(stream), ctx->pdl, cta, w->glu, nullptr, 0,
                                        nullptr, 0, static_cast<const uint32_t*>(own_flags), nranks);
  if (e != cudaSuccess) return cuda_fail(e, "gathered tc gemm launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_matmul_gather(s4_ctx* ctx, const s4_weight* w, const void* x, int ldx, int M, void* const* dst, int ndst,
                     int ldy, int col0, void* stream) {
  return matmul_gather_impl(ctx, w, x, ldx, M, dst, ndst, ldy, col0, nullptr, 0, stream);
}

int s4_matmul_gather_wait(s4_ctx* ctx, const s4_weight* w, const void* x, int ldx, int M, void* const* dst,
                          int ndst, int ldy, int col0, const void* own_flags, int nranks, void* stream) {
  if (!own_flags) return fail(S4_ERR_INVALID, "NULL flag array");
  return matmul_gather_impl(ctx, w, x, ldx, M, dst, ndst, ldy, col0, own_flags, nranks, stream);
}

int s4_silu_mul_gather(s4_ctx* ctx, const void* big, int M, int Is, void* const* dst, int ndst, int ldd, int col0,
                       void* stream) {
  if (!ctx || !big || !dst) return fail(S4_ERR_INVALID, "NULL argument");
  if (M < 0 || Is < 8) return fail(S4_ERR_INVALID, "bad shape");
  if (M == 0) return S4_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_silu_mul_gather(static_cast<const __half*>(big), M, Is,
                                             reinterpret_cast<__half* const*>(dst), ndst, ldd, col0, ctx->sm_count,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "silu_mul_gather launch (Is, ldd, col0 must be multiples of 8)");
  ++ctx->launches;
  return S4_OK;
}

int s4_peer_barrier(s4_ctx* ctx, void* const* flags, int nranks, int rank, uint32_t epoch, void* stream) {
  if (!ctx || !flags) return fail(S4_ERR_INVALID, "NULL argument");
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return fail(S4_ERR_INVALID, "bad rank / nranks");
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_peer_barrier(reinterpret_cast<uint32_t* const*>(flags), nranks, rank, epoch, ctx->err,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "peer barrier launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_peer_signal(s4_ctx* ctx, void* const* flags, int nranks, int rank, void* stream) {
  if (!ctx || !flags) return fail(S4_ERR_INVALID, "NULL argument");
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return fail(S4_ERR_INVALID, "bad rank / nranks");
  for (int q = 0; q < nranks; ++q)
    if (!flags[q]) return fail(S4_ERR_INVALID, "NULL flag array of rank %d", q);
  DeviceGuard guard(ctx->device);
  cudaError_t e = s4::launch_peer_signal(reinterpret_cast<uint32_t* const*>(flags), nranks, rank,
                                         static_cast<cudaStream_t>(stream), ctx->pdl);
  if (e != cudaSuccess) return cuda_fail(e, "peer signal launch");
  ++ctx->launches;
  return S4_OK;
}

int s4_plan(s4_ctx* ctx, int M, int N, int K, int* family, int* tile, int* split) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  if (M < 1) M = 1;
  const Bucket b = choose(ctx, M, N, K);
  int t = b.tile, g = b.split;
  if (b.family == S4_FAMILY_TC && N > 0 && K > 0) {
    // the tile and CTA count the call would launch with
    s4_weight w;
    w.N = N;
    w.K = K;
    w.nblk = (N + s4::kRowsPerBlock - 1) / s4::kRowsPerBlock;
    w.ktiles = (K + s4::kKPerTile - 1) / s4::kKPerTile;
    int tn = t, grid = ctx->sm_count;
    if (tn == 0) auto_shape(M, &w, ctx->sm_count, &tn, &grid);
    if (g > 0) grid = std::min(g, ctx->sm_count);
    t = tn;
    g = grid;
  }
  if (family) *family = b.family;
  if (tile) *tile = t;
  if (split) *split = g;
  return S4_OK;
}

int s4_force(s4_ctx* ctx, int family, int tile, int split) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  if (family != S4_FAMILY_AUTO && family != S4_FAMILY_GEMV && family != S4_FAMILY_TC)
    return fail(S4_ERR_INVALID, "unknown family %d", family);
  if (family == S4_FAMILY_TC && !s4::tc_available()) return fail(S4_ERR_UNSUPPORTED, "tc family is not built");
  if (tile < 0 || split < 0) return fail(S4_ERR_INVALID, "tile and split must be >= 0");
  if (family == S4_FAMILY_GEMV && split > s4::gemv_max_split())
    return fail(S4_ERR_INVALID, "GEMV split %d exceeds %d", split, s4::gemv_max_split());
  ctx->forced = Bucket{INT_MAX, family, tile, split, s4::kFixupAuto, 0, 0};
  return S4_OK;
}

int s4_set_table(s4_ctx* ctx, const char* json) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL argument");
  std::vector<Bucket> t;
  std::string why;
  try {
    if (!json) {
      ctx->table = default_table();  // back to the built-in table
      return S4_OK;
    }
    if (!parse_table(json, t, why)) return fail(S4_ERR_INVALID, "dispatch table: %s", why.c_str());
  } catch (const std::bad_alloc&) {
    return fail(S4_ERR_NOMEM, "dispatch table: out of host memory");
  }
  for (const Bucket& b : t)
    if (b.family == S4_FAMILY_GEMV && b.split > s4::gemv_max_split())
      return fail(S4_ERR_INVALID, "GEMV split %d exceeds %d", b.split, s4::gemv_max_split());
  ctx->table = t;
  return S4_OK;
}

int s4_check_errors(s4_ctx* ctx, uint32_t* flags) {
  if (!ctx || !flags) return fail(S4_ERR_INVALID, "NULL argument");
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(flags, ctx->err, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "error word read");
  return S4_OK;
}

int s4_clear_errors(s4_ctx* ctx) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(ctx->tickets, 0, kMaxTickets * sizeof(uint32_t));
  if (e != cudaSuccess) return cuda_fail(e, "error reset");
  return S4_OK;
}

int s4_launch_count(s4_ctx* ctx, uint64_t* count) {
  if (!ctx || !count) return fail(S4_ERR_INVALID, "NULL argument");
  *count = ctx->launches;
  return S4_OK;
}

int s4_device_info(s4_ctx* ctx, int* device, int* sm_count) {
  if (!ctx) return fail(S4_ERR_INVALID, "NULL context");
  if (device) *device = ctx->device;
  if (sm_count) *sm_count = ctx->sm_count;
  return S4_OK;
}

}  // extern "C"
