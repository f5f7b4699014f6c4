/*
 * s4mm — B200 (sm_100a) int4 MatMulNBits linear path, C ABI.
 *
 * Weight format (what the reference's engine uploads, convert/export_engine.py:3-4,17-26):
 *   packed  uint8  [N][K/32][16]   element 2i of a 32-block in the low nibble of byte i,
 *                                  element 2i+1 in the high nibble, value q means q-8;
 *   scales  fp16   [N][K/32]       one per block, any sign.
 * Matmul:  y[M][N] (fp16) = x[M][K] (fp16) @ ((q-8)*scale)^T, fp32 accumulation.
 *
 * Every call returns an int status (S4_OK == 0). On failure s4_last_error() gives a message
 * for the calling thread. No call throws, none aborts the process.
 *
 * Threading: a context is bound to one device; it is thread-compatible, not thread-safe
 * (one host thread drives it at a time), like the reference's single inference worker
 * (web/public/js/worker.js:249-252). Work is asynchronous on the stream passed in unless a
 * function says it is synchronous.
 */
#ifndef S4MM_H
#define S4MM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define S4_API __attribute__((visibility("default")))
#else
#define S4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define S4_OK 0
#define S4_ERR_INVALID 1      /* bad argument: null pointer, size, alignment */
#define S4_ERR_CUDA 2         /* a CUDA runtime call failed */
#define S4_ERR_NOMEM 3        /* device or pinned memory allocation failed */
#define S4_ERR_DEVICE 4       /* a kernel reported an error (bounded wait expired) */
#define S4_ERR_UNSUPPORTED 5  /* no sm_100 device, or shape outside what a kernel handles */
#define S4_ERR_IO 6           /* a cache file is missing, unreadable, or not a weight of this layout */

/* Kernel families of the dispatcher (s4_force / s4_plan). */
#define S4_FAMILY_AUTO 0
#define S4_FAMILY_GEMV 1      /* decode GEMV, M <= 16: cluster split-K over the weight bytes */
#define S4_FAMILY_TC 2        /* tcgen05 GEMM, weights dequantised to fp16 in shared memory */

typedef struct s4_ctx s4_ctx;
typedef struct s4_weight s4_weight;
typedef struct s4_chain s4_chain;
typedef struct s4_manifest s4_manifest;

/* Library version, (major << 16) | minor. */
S4_API int s4_version(void);

/* Message of the last failed call on this thread ("" if none). */
S4_API const char* s4_last_error(void);

/* Open a context on CUDA device `device`. Replaces the device side of Engine.create
 * (web/public/engine/engine.js:63-87): the context owns the split-K scratch the reference
 * allocates per activation pool (engine.js:190-199) and the dispatch table. */
S4_API int s4_init(int device, s4_ctx** out);
/* Close a context. Its weights and chains are not freed with it: s4_weight_free / s4_chain_free
 * stay valid on them afterwards (in either order), every other call on them needs the context. */
S4_API int s4_destroy(s4_ctx* ctx);

/* Upload one fused projection's int4 weight from HOST memory and repack it on the device into
 * the B200 tiled layout. Synchronous: the weight is usable on any stream when it returns.
 * Replaces the Gemm constructor's upload (web/public/gemmbench/kernels.js:84-87) and the
 * engine's shard writes (engine.js:76-84). N >= 1 (any N; padded internally), K % 32 == 0.
 * flags: 0 (reserved). */
S4_API int s4_weight_upload(s4_ctx* ctx, const uint8_t* packed, const uint16_t* scales, int N, int K,
                     uint32_t flags, s4_weight** out);

/* Same, from DEVICE pointers already holding the MatMulNBits bytes (a shard range resolved like
 * the engine's w(name), engine.js:175-180). Synchronous. */
S4_API int s4_weight_upload_device(s4_ctx* ctx, const void* packed_dev, const void* scales_dev, int N,
                            int K, uint32_t flags, s4_weight** out);

/* Download-format ("wire") scales: N row headers of 4 bytes (m = fp16 bits, j = u16, little-endian)
 * then N*G codes sign << 7 | k, decoded to fp16 toHalf(fromHalf(m) * 2^(-k*j/4096)) | sign << 15 as
 * web/public/engine/wire.js:5-33 does (decodeScales), bit for bit, on the device. wire_dev holds
 * 4*N + N*G bytes (any alignment); scales_dev receives N*G fp16 (2-byte aligned). Stream-ordered
 * and allocation-free except the context's first wire call, which uploads a 32 KB table (do that
 * call outside stream capture). Replaces decodeScales in unpackShard (wire.js:37-46, engine.js:82)
 * and putRows (engine.js:128-136, one row per call there, N rows per call here). */
S4_API int s4_decode_wire_scales(s4_ctx* ctx, const void* wire_dev, int N, int G, void* scales_dev,
                                 void* stream);

/* s4_weight_upload with the scales in the wire format (4*N + N*(K/32) bytes of host memory):
 * uploads, decodes on the device and repacks. Synchronous. */
S4_API int s4_weight_upload_wire(s4_ctx* ctx, const uint8_t* packed, const uint8_t* wire_scales, int N, int K,
                                 uint32_t flags, s4_weight** out);

/* Non-default weight formats (web/public/gemmbench/kernels.js:5-12; a tensor's format is
 * {bits, group, asym}, engine.js:36 fmtOf). A block of 32 consecutive K values of one row takes
 * `bits` u32 words: 4 bits: element e at bits 4(e%8) of word e/8; 2 bits: element e at bits 2(e%16)
 * of word e/16; 3 bits: words 0-1 the low two bits as in the 2-bit layout, bit e of word 2 the high
 * bit. q: [N][K/32][bits] u32; scales: fp16 [N][K/group], group 32 or 64, K % group == 0.
 * Symmetric: w = (q - 2^(bits-1)) * scale. bias: fp16 [N][K/group] for the asymmetric form
 * w = q * scale + bias, or NULL. flags: S4_UPLOAD_DEVICE when q/scales/bias are device pointers,
 * else host memory. Synchronous. 4-bit group-32 symmetric is s4_weight_upload. Symmetric formats
 * become plain int4 weights (exactly); asymmetric ones keep their biases and run through s4_matmul and
 * s4_matmul_noalloc (the chained launch rejects them with S4_ERR_UNSUPPORTED). */
#define S4_UPLOAD_DEVICE 1u
/* Symmetric 2-bit weights only: also keep the weight in a native 2-bit decode layout (2048 bytes per
 * 128 x 64 chunk instead of 4096), which the decode GEMV (M <= 16, s4_matmul) streams instead of the
 * int4 layout; the tcgen05 GEMM and chained runs keep reading the int4 layout, so the weight takes
 * 1.44x the device memory. Results are identical (the same fp16 fragments enter the same MMAs). A
 * single decode call is dominated by launch and first-byte latency, so it gains little time (measured
 * within 3 % on B200); no counterpart in the reference, whose shaders read the 2-bit words in place.
 * s4_weight_save stores the int4 layout only: a weight loaded back decodes from it. */
#define S4_UPLOAD_DECODE_LAYOUT 2u
S4_API int s4_weight_upload_format(s4_ctx* ctx, const void* q, const void* scales, const void* bias, int N, int K,
                                   int bits, int group, uint32_t flags, s4_weight** out);

/* A fused gate|up projection whose matmul writes the SiLU*mul of its two halves: packed / scales are
 * the MatMulNBits bytes of the [2I][K] weight (rows 0..I-1 gate, I..2I-1 up, the engine's fused
 * layout), and s4_matmul / s4_matmul_gather on it write y[M][I] = silu(x W_gate^T) * (x W_up^T)
 * (the SILU_MUL step, wgsl.js:81-90, engine.js:279-280, done in the GEMM epilogue; gate and up are
 * rounded to fp16 first, as when they pass through memory). I % 64 == 0. Upload permutes rows so a
 * 128-row tile holds 64 gate rows and their 64 up rows. s4_weight_info reports N = I. Not usable by a
 * chain or s4_matmul_noalloc (S4_ERR_UNSUPPORTED). flags: S4_UPLOAD_DEVICE for device pointers.
 * Synchronous. */
S4_API int s4_weight_upload_glu(s4_ctx* ctx, const void* packed, const void* scales, int I, int K, uint32_t flags,
                                s4_weight** out);

S4_API int s4_weight_free(s4_weight* w);

/* Weight manifest of an exported engine: the JSON the exporter writes (convert/export_engine.py:29-34,
 * 83-85), "shards": [{"path", "start", "bytes"}] laid out back to back from global offset 0 and
 * "tensors": {name: {"offset", "bytes", "dtype", "shape", "N", "K"}} with global offsets. Parsing and
 * lookups are host-only (no device, no context). s4_manifest_tensor is the engine's w(name)
 * (web/public/engine/engine.js:175-180): the shard holding the tensor and the byte offset inside it
 * (S4_ERR_INVALID "no tensor <name>" when absent, engine.js:177), its size, and N / K for a quantised
 * projection's ".q" tensor (-1 otherwise). s4_manifest_shard gives a shard's path (valid while the
 * manifest lives) and size. */
S4_API int s4_manifest_open(const char* json, s4_manifest** out);
S4_API int s4_manifest_free(s4_manifest* m);
S4_API int s4_manifest_counts(const s4_manifest* m, int* nshards, int* ntensors);
S4_API int s4_manifest_shard(const s4_manifest* m, int i, const char** path, size_t* bytes);
S4_API int s4_manifest_tensor(const s4_manifest* m, const char* name, int* shard, size_t* offset, size_t* bytes,
                              int* N, int* K);

/* Upload the quantised projection `name` (the pair name.q / name.s of the manifest, N = the exported,
 * 64-row padded N) from the engine's shard buffers: shards[i] is shard i's bytes, in host memory, or in
 * device memory with flags = S4_UPLOAD_DEVICE (a device range must leave name.q 4-byte and name.s
 * 2-byte aligned). Checks dtypes and sizes against N and K, then runs s4_weight_upload /
 * s4_weight_upload_device. Replaces the shard upload + w(name) binding of a projection in
 * Engine.create / plan() (engine.js:76-84, 175-180, 239). Synchronous. */
S4_API int s4_weight_upload_named(s4_ctx* ctx, const s4_manifest* m, const void* const* shards, const char* name,
                                  uint32_t flags, s4_weight** out);

/* On-disk cache of repacked weights (the role of the worker's OPFS asset cache, worker.js:27-44,
 * 82-100, here holding the device layout so a later load skips decode and repack). A file is a
 * 64-byte header (magic "S4WL", layout version, N, K, asymmetric flag, section sizes, a 64-bit
 * checksum of the payload) followed by the device layout. Entries are keyed by the caller's file
 * name (the host side builds names with the worker's fingerprint prefix). Synchronous.
 * s4_weight_load returns S4_ERR_IO for a missing, truncated or corrupt file, or one written by a
 * different layout version; the caller then uploads from the shard and saves again. */
S4_API int s4_weight_save(const s4_weight* w, const char* path);
S4_API int s4_weight_load(s4_ctx* ctx, const char* path, s4_weight** out);

/* Shape and device footprint of an uploaded weight. */
S4_API int s4_weight_info(const s4_weight* w, int* N, int* K, size_t* device_bytes);

/* Copy the repacked device layout back to host buffers (diagnostics and round-trip tests).
 * wq_bytes / ws_bytes must be at least what s4_weight_layout_bytes reports. Synchronous. */
S4_API int s4_weight_layout_bytes(const s4_weight* w, size_t* wq_bytes, size_t* ws_bytes);
S4_API int s4_weight_download_layout(const s4_weight* w, void* wq_host, size_t wq_bytes, void* ws_host,
                              size_t ws_bytes);

/* y[M][N] = x[M][K] @ W^T on DEVICE pointers, asynchronous on `stream` (a cudaStream_t, NULL =
 * legacy default stream). x and y are fp16 row-major with row strides K and N, 16-byte aligned.
 * Allocates nothing. Replaces plan().matmul(A, wname, Y) (engine.js:236-246) including the
 * split-K REDUCE step (kernels.js:269-282, engine.js:244). M == 0 is a no-op. */
S4_API int s4_matmul(s4_ctx* ctx, const s4_weight* w, const void* x, int M, void* y, void* stream);

/* The standalone Gemm object's setA + encode + readY on HOST buffers (kernels.js:90-103):
 * copies x to the device, runs s4_matmul, copies y back. Synchronous. Uses context-owned
 * staging buffers that grow on demand. */
S4_API int s4_matmul_host(s4_ctx* ctx, const s4_weight* w, const uint16_t* x, int M, uint16_t* y);

/* Asynchronous form of s4_matmul_host on `stream`: host->device copy of x, matmul, device->host
 * copy of y, nothing waited for (the encode() + mapAsync half of Gemm, kernels.js:98-103).
 * x and y should be pinned host memory; they must stay valid until the stream reaches this
 * work. Calls on one context share its staging buffers, so keep them on one stream. */
S4_API int s4_matmul_host_async(s4_ctx* ctx, const s4_weight* w, const uint16_t* x, int M, uint16_t* y,
                                void* stream);

/* y[M][N] = x[M][K] @ W^T like s4_matmul, for callers that cannot allocate device memory when they
 * run a matmul (a host whose memory manager already owns the whole device, or a serving loop that
 * must not take cudaMalloc's implicit device synchronisation). It needs no context-owned scratch:
 * the tcgen05 split-K GEMM keeps its partials, tile counters and error word in one static 8 MiB
 * device array that every GPU loading this library holds until exit. It calls no allocator. It needs
 * no live context either: the weight records its device and SM count, so it may be called after
 * s4_destroy of the context the weight was uploaded with. Limit: ceil(M/256) * ceil(N/128) <= 16384
 * (larger calls are rejected with S4_ERR_INVALID); the CTA count is a divisor of the tile count between
 * half the SMs and all of them when there is one (whole tiles, no partials), else the SM count capped so
 * that each CTA's two partial slots of (M rounded up to 16, at most 256) x 128 fp32 fit the array (31
 * CTAs at M >= 256, all 148 SMs at M <= 48). The first call on a device looks up the array's device address
 * (do it before any stream capture; a cudaDeviceReset of that device leaves the looked-up address
 * stale, so do not reset a device this library has used). All calls share the array: calls that
 * overlap on the GPU race. A bounded wait that expires sets the array's error word, which stays set
 * until s4_noalloc_check_errors clears it. No counterpart in the reference. DEVICE pointers,
 * asynchronous on `stream`. */
S4_API int s4_matmul_noalloc(const s4_weight* w, const void* x, int M, void* y, void* stream);
/* Error word of s4_matmul_noalloc's static scratch on `device` (0 = clean; the bits of
 * s4_check_errors), read after a device synchronisation; clear != 0 resets it. Allocates nothing.
 * No counterpart in the reference. */
S4_API int s4_noalloc_check_errors(int device, uint32_t* flags, int clear);

/* Chained decode GEMV: a fixed list of matmuls y_i[M_i][N_i] = x_i @ W_i^T (1 <= M_i <= 16) run by ONE
 * persistent launch, like the engine's recorded step list submitted at once (plan(), engine.js:236-282).
 * The weights of later ops stream into shared memory while earlier ops finish, so a decode step's GEMVs
 * move weight bytes back to back instead of paying a launch and a DRAM ramp each. dep[i] is the index
 * of an earlier op whose output op i reads (its x_i aliases y_dep), or -1; dep may be NULL (all -1).
 * Buffers are bound at creation (DEVICE pointers, x 16-byte aligned) and must stay valid while the
 * chain is used; results equal s4_matmul's within fp32 summation order. s4_chain_run is asynchronous
 * on `stream`; runs of one chain must not overlap. Creation is synchronous and allocates the chain's
 * split-K scratch. S4_ERR_UNSUPPORTED if an op's activation window does not fit in shared memory.
 * s4_chain_run launches as a programmatic dependent launch: a run that follows another kernel on the
 * same stream streams its weights while that kernel drains (it reads activations and scratch only
 * after that kernel completes). Its CTAs wait on one another, so chained runs issued on DIFFERENT
 * streams must not execute concurrently with it (environment S4_PDL=0 gives a cooperative launch,
 * safe on any streams). s4_chain_run_host always launches cooperatively. */
S4_API int s4_chain_create(s4_ctx* ctx, int nops, const s4_weight* const* w, const void* const* x, void* const* y,
                           const int* M, const int* dep, s4_chain** out);
S4_API int s4_chain_run(s4_ctx* ctx, s4_chain* chain, void* stream);
/* Host-buffer form (the engine's write inputs / submit / read outputs): copies x_bytes from HOST
 * x_host to DEVICE x_dev, runs the chain, copies y_bytes from DEVICE y_dev to HOST y_host, all on
 * `stream`, nothing waited for. The chain's bound inputs must lie in [x_dev, x_dev + x_bytes) and its
 * outputs of interest in [y_dev, y_dev + y_bytes); host buffers should be pinned and stay valid until
 * the stream reaches this work. */
S4_API int s4_chain_run_host(s4_ctx* ctx, s4_chain* chain, const void* x_host, void* x_dev, size_t x_bytes,
                             void* y_host, const void* y_dev, size_t y_bytes, void* stream);
S4_API int s4_chain_info(const s4_chain* chain, int* grid, int* slots, int* smem_bytes);
S4_API int s4_chain_free(s4_chain* chain);

/* mid[M][I] = silu(big[:, :I]) * big[:, I:2I], fp16 in/out, fp32 math, DEVICE pointers,
 * asynchronous. Replaces SILU_MUL (web/public/engine/wgsl.js:81-90). */
S4_API int s4_silu_mul(s4_ctx* ctx, const void* big, int M, int I, void* mid, void* stream);

/* Residual add + RMSNorm between projections (ADD_NORM, web/public/engine/wgsl.js:55-78):
 * x[M][D] fp32 residual stream, updated in place by x += y when y (fp16) is not NULL; then
 * h[M][D] = f16(x * rsqrt(mean(x^2) + eps) * w), w fp32 [D] (the stored 1 + weight) or NULL for
 * ones. DEVICE pointers, asynchronous. */
S4_API int s4_add_rmsnorm(s4_ctx* ctx, float* x, const void* y, const float* w, int M, int D, float eps, void* h,
                          void* stream);

/* A projection followed by ADD_NORM in one call (out_proj / o_proj / down then post_norm / in_norm,
 * web/public/engine/engine.js:247, 277; wgsl.js:55-78): y = x @ W^T is never stored; instead
 * resid[M][N] (fp32, updated in place) += f16(y) and h[M][N] = f16(resid * rsqrt(mean(resid^2) + eps)
 * * norm_w), norm_w fp32 [N] (the stored 1 + weight) or NULL for ones. On the tcgen05 path (N a
 * multiple of 32) the residual add and the row sums of squares run in the GEMM's epilogue and one
 * row kernel normalises; on the GEMV path y goes through h and is normalised in place. x [M][K] fp16.
 * Not for fused gate|up weights. DEVICE pointers, 16-byte aligned; asynchronous on `stream`. Uses the
 * context's scratch, so calls on one context must not overlap on the GPU. */
S4_API int s4_matmul_add_rmsnorm(s4_ctx* ctx, const s4_weight* w, const void* x, int M, float* resid,
                                 const float* norm_w, float eps, void* h, void* stream);

/* Online input rotation of a tensor exported with `had: n` (engine.js:238, wgsl.js:94-110): every
 * contiguous n-block of a[M][K] (fp16, K % n == 0, n a power of two in [2, 32768]) is replaced in place
 * by its orthonormal Walsh-Hadamard transform, computed in fp32 with the shader's butterfly order and
 * rounded to fp16 once. Run it on the matmul's input before s4_matmul. DEVICE pointer, asynchronous. */
S4_API int s4_fwht(s4_ctx* ctx, void* a, int M, int K, int n, void* stream);

/* ---- column-sharded prefill over NVLink (one process per GPU on one node) ----
 * Each rank computes an N/g slice of every projection and writes it straight into every rank's
 * gathered output buffer through peer mappings (the all-gather fused into the GEMM epilogue; the
 * north star's NCCL all-gather of outputs, engine calls engine.js:257-281, sharded). */

/* A device buffer of its own cudaMalloc allocation, so that peers can map it (s4_ipc_*). Zeroed. */
S4_API int s4_buffer_alloc(s4_ctx* ctx, size_t bytes, void** ptr);
S4_API int s4_buffer_free(s4_ctx* ctx, void* ptr);

/* CUDA IPC: export a buffer from s4_buffer_alloc as a 64-byte handle; map a peer's handle on the
 * context's device; unmap. Plain peer mappings (no multicast objects). */
S4_API int s4_ipc_handle(s4_ctx* ctx, const void* ptr, void* handle64);
S4_API int s4_ipc_open(s4_ctx* ctx, const void* handle64, void** ptr);
S4_API int s4_ipc_close(s4_ctx* ctx, void* ptr);

/* y = x @ W^T (tcgen05 GEMM) with x of row stride ldx (elements, ldx >= K, ldx*2 % 16 == 0), the
 * result written to each of ndst (<= 8) buffers at dst[d][m * ldy + col0 + n] (this rank's column
 * slice of every rank's gathered buffer; the pointers may be peer mappings). Asynchronous. */
S4_API int s4_matmul_gather(s4_ctx* ctx, const s4_weight* w, const void* x, int ldx, int M, void* const* dst,
                            int ndst, int ldy, int col0, void* stream);

/* SiLU*mul of this rank's gate|up slice big[M][2*Is] written to dst[d][m * ldd + col0 + j]
 * (Is, ldd, col0 multiples of 8; 16-byte aligned buffers). Asynchronous. */
S4_API int s4_silu_mul_gather(s4_ctx* ctx, const void* big, int M, int Is, void* const* dst, int ndst, int ldd,
                              int col0, void* stream);

/* Barrier across nranks GPUs: flags[q] is rank q's flag array (>= 16 uint32, zeroed, peer-mapped);
 * every rank passes the same increasing epoch, or every rank passes 0 on every call: the epoch is
 * then counted on the device (slot 8 of the rank's own array), so the barrier can be captured in
 * a CUDA graph and replayed. Do not mix the two forms on one flag array. A wait that exceeds 1 s
 * sets the context's error word (s4_check_errors) instead of hanging. Asynchronous on `stream`. */
S4_API int s4_peer_barrier(s4_ctx* ctx, void* const* flags, int nranks, int rank, uint32_t epoch, void* stream);

/* The barrier split in two, so its wait overlaps the next kernel's start. s4_peer_signal: once the
 * work before it on `stream` has finished (its peer stores included), count the next epoch on the
 * device (slot 8 of this rank's array, as s4_peer_barrier with epoch 0) and store it into every rank's
 * array (flags as for s4_peer_barrier). The consumers of the gathered data then wait themselves:
 * s4_matmul_gather_wait (its activation loads wait; the weight stream starts at once) and
 * s4_add_rmsnorm_wait take this rank's own flag array and wait until all nranks ranks have signalled
 * this rank's latest epoch. Every rank signals the same number of times. A wait past 1 s sets the
 * context's error word. No counterpart in the reference (its engine runs on one GPU); it replaces the
 * all-gather step of the column-sharded prefill. Asynchronous on `stream`. */
S4_API int s4_peer_signal(s4_ctx* ctx, void* const* flags, int nranks, int rank, void* stream);
S4_API int s4_matmul_gather_wait(s4_ctx* ctx, const s4_weight* w, const void* x, int ldx, int M, void* const* dst,
                                 int ndst, int ldy, int col0, const void* own_flags, int nranks, void* stream);
S4_API int s4_add_rmsnorm_wait(s4_ctx* ctx, float* x, const void* y, const float* w, int M, int D, float eps,
                               void* h, const void* own_flags, int nranks, void* stream);

/* Dispatcher. s4_plan reports the (family, tile, split) s4_matmul will use for M on an
 * (N, K) weight (for the tcgen05 family with N and K given: the tokens per tile and CTAs it launches;
 * otherwise the bucket's values, 0 = kernel default); replaces matmulKernel(M) (engine.js:17-33).
 * s4_force pins a choice for every later call (family 0 = back to the table), like matmulKernel's
 * `force` (engine.js:23); tile/split 0 mean "kernel default". s4_set_table loads a measured M-bucket
 * table (the role of the tile table tune.html produces, engine/tune.html:8-24):
 * JSON {"buckets": [{"max_m": int, "family": "gemv"|"tc", "tile": int, "split": int,
 * "fixup": "auto"|"kernel"|"cta", "K": int, "N": int}, ...]}. A call uses the first bucket whose max_m
 * covers M and whose K and N (weight columns and rows, 0 or absent = any) match its weight; GEMV split =
 * CTAs per n-block, tcgen05 split = CTAs, fixup = who sums split tiles (a second kernel or their last
 * CTA). The last bucket without K and N covers every larger M. json == NULL restores the built-in
 * table (the measured table compiled into the library). */
S4_API int s4_plan(s4_ctx* ctx, int M, int N, int K, int* family, int* tile, int* split);
S4_API int s4_force(s4_ctx* ctx, int family, int tile, int split);
S4_API int s4_set_table(s4_ctx* ctx, const char* json);

/* Device-side error word written by kernels whose bounded waits expired; 0 = clean.
 * Reading it synchronises the context's device. s4_clear_errors resets it and the split-K
 * arrival counters. */
S4_API int s4_check_errors(s4_ctx* ctx, uint32_t* flags);
S4_API int s4_clear_errors(s4_ctx* ctx);

/* Number of kernels this context has launched since s4_init (host-side count). */
S4_API int s4_launch_count(s4_ctx* ctx, uint64_t* count);

/* Number of SMs and the device ordinal of the context. */
S4_API int s4_device_info(s4_ctx* ctx, int* device, int* sm_count);

#ifdef __cplusplus
}
#endif
#endif /* S4MM_H */
