// mla_capi.cu -- the C ABI of libkvl_mla_cuda: the reference runtime's MLA
// state / decode / prefill functions (include/kvl/mla_compressed_state.h,
// include/kvl/mla_compressed_q8_state.h, kvl_mla_prefill_bf16 of
// include/kvl/ops.h) served from GPU memory, plus the device-pointer entry
// points of include/kvl/mla_cuda.h.
//
// Conventions kept from the reference: every call validates its arguments in
// the reference's order and returns -1 without touching the state when a check
// fails (src/mla_compressed_state.c:92-98); decode appends the current token
// before attending; truncate/reset are O(1) on `len`; free zeroes the struct.
// CUDA failures also return -1.  There is no CPU fallback: without a usable
// GPU every compute call fails.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "attend_host.cuh"
#include "kvl/mla_compressed_q8_state.h"
#include "kvl/mla_compressed_state.h"
#include "kvl/mla_cuda.h"
#include "flash_prefill.cuh"
#include "gemm.cuh"
#include "mla_kernels.cuh"
#include "peer_merge.cuh"

#define KVL_EXPORT extern "C" __attribute__((visibility("default")))

namespace kvl {
namespace {

thread_local std::string g_err;

void set_err(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  static const bool verbose = [] {
    const char *v = getenv("KVL_CUDA_VERBOSE");
    return v && *v && *v != '0';
  }();
  if (verbose) fprintf(stderr, "kvl_mla_cuda: %s\n", buf);
}

#define CK(expr)                                                                        \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess) {                                                            \
      set_err("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return -1;                                                                        \
    }                                                                                   \
  } while (0)

struct DBuf {
  void *p = nullptr;
  size_t n = 0;
  bool ensure(size_t bytes) {
    if (bytes <= n) return true;
    cudaFree(p);
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return false;
    n = bytes;
    return true;
  }
  template <typename T>
  T *as() const { return static_cast<T *>(p); }
};

struct PBuf {  // pinned host staging
  void *p = nullptr;
  size_t n = 0;
  bool ensure(size_t bytes) {
    if (bytes <= n) return true;
    cudaFreeHost(p);
    p = nullptr;
    n = 0;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) return false;
    n = bytes;
    return true;
  }
  template <typename T>
  T *as() const { return static_cast<T *>(p); }
};

std::atomic<int> g_weight_cache{-1};

bool weight_cache_enabled() {
  int v = g_weight_cache.load();
  if (v < 0) {
    int en = 0;
    const char *a = getenv("KVL_CUDA_WEIGHT_CACHE");
    if (a && *a && *a != '0') en = 1;
    const char *t = getenv("KVL_TRUNK_CACHE_MIB");
    if (t && atol(t) >= 1706) en = 1;
    int expected = -1;
    g_weight_cache.compare_exchange_strong(expected, en);
    v = g_weight_cache.load();
  }
  return v == 1;
}

struct DevW {
  const uint16_t *q, *kva, *kvan, *kvb, *o;
};

constexpr int kMaxPrefillChunks = 8;

struct Ctx {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  // host-buffer prefill: copy streams and per-chunk events (created on first use)
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev_in[kMaxPrefillChunks] = {}, ev_out[kMaxPrefillChunks] = {};
  std::mutex mu;
  DBuf x, q, ka, qabs, mix, ho, y, rowf, kvtmp;
  DBuf wq, wkva, wkvan, wkvb, wo;  // per-call weight upload
  PBuf pin_io, pin_plan;
  DevicePlan plan;
  std::unordered_map<const void *, std::pair<size_t, void *>> wcache;
};

std::mutex g_ctx_mu;
std::unordered_map<int, Ctx *> g_ctx;

Ctx *get_ctx(int device) {
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  auto it = g_ctx.find(device);
  if (it != g_ctx.end()) return it->second;
  Ctx *c = new Ctx();
  c->device = device;
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    set_err("cannot open CUDA device %d", device);
    delete c;
    return nullptr;
  }
  cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device);
  g_ctx[device] = c;
  return c;
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) {
    set_err("no CUDA device available");
    return -1;
  }
  return d;
}

// One weight tensor on the device: cached by host pointer, or uploaded into a
// per-context buffer on every call.
int stage_weight(Ctx &c, DBuf &buf, const uint16_t *host, size_t elems, const uint16_t **dev) {
  const size_t bytes = elems * sizeof(uint16_t);
  if (weight_cache_enabled()) {
    auto it = c.wcache.find(host);
    if (it != c.wcache.end() && it->second.first == bytes) {
      *dev = static_cast<const uint16_t *>(it->second.second);
      return 0;
    }
    void *p = nullptr;
    CK(cudaMalloc(&p, bytes));
    CK(cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice));
    if (it != c.wcache.end()) cudaFree(it->second.second);
    c.wcache[host] = {bytes, p};
    *dev = static_cast<const uint16_t *>(p);
    return 0;
  }
  if (!buf.ensure(bytes)) {
    set_err("cudaMalloc of %zu weight bytes failed", bytes);
    return -1;
  }
  CK(cudaMemcpyAsync(buf.p, host, bytes, cudaMemcpyHostToDevice, c.stream));
  *dev = buf.as<const uint16_t>();
  return 0;
}

int stage_weights(Ctx &c, const KvlMlaConfig &cfg, const KvlMlaBF16 &w, DevW &d, bool need_q) {
  const size_t H = cfg.hidden_size, NH = cfg.num_heads, DN = cfg.qk_nope_dim, DR = cfg.qk_rope_dim;
  const size_t DV = cfg.v_head_dim, R = cfg.kv_lora_rank;
  d = DevW{nullptr, nullptr, nullptr, nullptr, nullptr};
  if (need_q) {
    if (stage_weight(c, c.wq, w.q_proj, NH * (DN + DR) * H, &d.q)) return -1;
    if (stage_weight(c, c.wkvb, w.kv_b_proj, NH * (DN + DV) * R, &d.kvb)) return -1;
    if (stage_weight(c, c.wo, w.o_proj, H * NH * DV, &d.o)) return -1;
  }
  if (stage_weight(c, c.wkva, w.kv_a_proj, (R + DR) * H, &d.kva)) return -1;
  if (stage_weight(c, c.wkvan, w.kv_a_norm, R, &d.kvan)) return -1;
  return 0;
}

// ------------------------------------------------------------------ states
enum Fmt { FMT_BF16 = 0, FMT_Q8 = 1 };

struct DevState {
  int fmt = FMT_BF16;
  int device = 0;
  int capacity = 0, cap_pad = 0, R = 0, DR = 0;
  int dev_len = 0;
  uint16_t *kv = nullptr;     // bf16 [cap_pad][R+DR]
  float *kvf = nullptr;       // fp32 [cap_pad][R+DR]: the rows the attend reads for shapes other
                              // than the production 16 x 512 x 64 (the reference's fp32 state)
  int8_t *lat8 = nullptr;     // q8 [cap_pad][R]
  float *lscale = nullptr;    // q8 [cap_pad]
  uint16_t *rope16 = nullptr; // q8 [cap_pad][DR]
  size_t bytes = 0;
  void release() {
    cudaFree(kv);
    cudaFree(kvf);
    cudaFree(lat8);
    cudaFree(lscale);
    cudaFree(rope16);
    kv = nullptr;
    kvf = nullptr;
    lat8 = nullptr;
    lscale = nullptr;
    rope16 = nullptr;
  }
};

std::mutex g_reg_mu;
std::unordered_map<const void *, DevState *> g_reg;  // key: host mirror pointer

DevState *find_state(const void *key) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(key);
  return it == g_reg.end() ? nullptr : it->second;
}

void register_state(const void *key, DevState *ds) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  g_reg[key] = ds;
}

DevState *unregister_state(const void *key) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(key);
  if (it == g_reg.end()) return nullptr;
  DevState *ds = it->second;
  g_reg.erase(it);
  return ds;
}

int alloc_dev_state(DevState &ds, int fmt, int capacity, int R, int DR, bool f32_rows = false) {
  ds.fmt = fmt;
  ds.capacity = capacity;
  ds.cap_pad = (capacity + kTileTok - 1) / kTileTok * kTileTok;
  ds.R = R;
  ds.DR = DR;
  ds.device = current_device();
  if (ds.device < 0) return -1;
  const size_t rows = ds.cap_pad;
  if (fmt == FMT_BF16) {
    ds.bytes = rows * (R + DR) * sizeof(uint16_t);
    CK(cudaMalloc(&ds.kv, ds.bytes));
    CK(cudaMemset(ds.kv, 0, ds.bytes));
    if (f32_rows) {
      const size_t fb = rows * (R + DR) * sizeof(float);
      CK(cudaMalloc(&ds.kvf, fb));
      CK(cudaMemset(ds.kvf, 0, fb));
      ds.bytes += fb;
    }
  } else {
    CK(cudaMalloc(&ds.lat8, rows * R));
    CK(cudaMalloc(&ds.lscale, rows * sizeof(float)));
    CK(cudaMalloc(&ds.rope16, rows * DR * sizeof(uint16_t)));
    CK(cudaMemset(ds.lat8, 0, rows * R));
    CK(cudaMemset(ds.lscale, 0, rows * sizeof(float)));
    CK(cudaMemset(ds.rope16, 0, rows * DR * sizeof(uint16_t)));
    ds.bytes = rows * (R + sizeof(float) + DR * sizeof(uint16_t));
  }
  return 0;
}

// Brings the device rows in line with the host struct: rows the caller wrote
// into the mirrors and published by raising `len` are uploaded; a lower `len`
// truncates.
int sync_bf16_state(Ctx &c, DevState &ds, const KvlMlaCompressedState &st) {
  if (st.len < ds.dev_len) {
    ds.dev_len = st.len;
    return 0;
  }
  if (st.len == ds.dev_len) return 0;
  const int n = st.len - ds.dev_len, R = ds.R, DR = ds.DR;
  if (!c.kvtmp.ensure(static_cast<size_t>(n) * (R + DR) * sizeof(float))) {
    set_err("cudaMalloc failed while uploading host rows");
    return -1;
  }
  float *tmp = c.kvtmp.as<float>();
  CK(cudaMemcpy2DAsync(tmp, (R + DR) * sizeof(float), st.latent + static_cast<size_t>(ds.dev_len) * R,
                       R * sizeof(float), R * sizeof(float), n, cudaMemcpyHostToDevice, c.stream));
  CK(cudaMemcpy2DAsync(tmp + R, (R + DR) * sizeof(float), st.rope + static_cast<size_t>(ds.dev_len) * DR,
                       DR * sizeof(float), DR * sizeof(float), n, cudaMemcpyHostToDevice, c.stream));
  CK(f32_to_bf16(ds.kv + static_cast<size_t>(ds.dev_len) * (R + DR), tmp, static_cast<long long>(n) * (R + DR),
                 c.stream));
  if (ds.kvf)
    CK(cudaMemcpyAsync(ds.kvf + static_cast<size_t>(ds.dev_len) * (R + DR), tmp,
                       static_cast<size_t>(n) * (R + DR) * sizeof(float), cudaMemcpyDeviceToDevice, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  ds.dev_len = st.len;
  return 0;
}

int sync_q8_state(Ctx &c, DevState &ds, const KvlMlaCompressedQ8State &st) {
  if (st.len < ds.dev_len) {
    ds.dev_len = st.len;
    return 0;
  }
  if (st.len == ds.dev_len) return 0;
  const size_t a = ds.dev_len, n = st.len - ds.dev_len, R = ds.R, DR = ds.DR;
  CK(cudaMemcpyAsync(ds.lat8 + a * R, st.latent_q8 + a * R, n * R, cudaMemcpyHostToDevice, c.stream));
  CK(cudaMemcpyAsync(ds.lscale + a, st.latent_scale + a, n * sizeof(float), cudaMemcpyHostToDevice, c.stream));
  CK(cudaMemcpyAsync(ds.rope16 + a * DR, st.rope_bf16 + a * DR, n * DR * sizeof(uint16_t),
                     cudaMemcpyHostToDevice, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  ds.dev_len = st.len;
  return 0;
}

bool cfg_dims_ok(const KvlMlaConfig &c) {
  return c.hidden_size > 0 && c.num_heads > 0 && c.qk_nope_dim > 0 && c.qk_rope_dim > 0 &&
         (c.qk_rope_dim & 1) == 0 && c.v_head_dim > 0 && c.kv_lora_rank > 0 && c.rope_theta > 0.0f;
}

// Attends the single-sequence plan [0, L) of a state into c.mix.
// The single-sequence plan of a state of L rows, uploaded on the call's stream.
int plan_state(Ctx &c, const DevState &ds, int L, int nh) {
  HostPlan hp;
  const long long row0 = 0;
  if (build_attend_plan(hp, 1, &L, &row0, c.sms) != 0) {
    set_err("attend plan failed (L=%d)", L);
    return -1;
  }
  if (!c.pin_plan.ensure(64 * 1024) ||
      c.plan.upload(hp, nh, ds.R, c.stream, c.pin_plan.p, c.pin_plan.n) != 0) {
    set_err("attend plan upload failed");
    return -1;
  }
  return 0;
}

// The attend of a state over the plan plan_state() uploaded.  q_dependent: the
// previous kernel on the stream is the absorb kernel that writes the query.
int attend_state(Ctx &c, const DevState &ds, int nh, float scale, bool q_dependent) {
  AttendLaunch a;
  a.q8 = ds.fmt == FMT_Q8;
  a.nh = nh;
  a.R = ds.R;
  a.DR = ds.DR;
  a.rows = ds.cap_pad;
  a.q = c.qabs.as<float>();
  a.out = c.mix.as<float>();
  a.kv = ds.kv;
  a.kvf = ds.kvf;
  a.lat8 = ds.lat8;
  a.lscale = ds.lscale;
  a.rope16 = ds.rope16;
  a.softmax_scale = scale;
  a.q_dependent = q_dependent;
  if (c.plan.launch(a, c.stream) != 0) {
    set_err("attend launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  return 0;
}

// One decode step of one token against a device state (both formats).
// Host x[H] -> host out[H]; the appended row is mirrored into the host arrays
// through the callback target pointers.
int decode_one(Ctx &c, DevState &ds, const KvlMlaConfig &cfg, const DevW &W, const float *x, float *out,
               int position, float *mir_lat, float *mir_rope, int8_t *mir_q8, float *mir_scale,
               uint16_t *mir_rope16) {
  const int H = cfg.hidden_size, NH = cfg.num_heads, DN = cfg.qk_nope_dim, DR = cfg.qk_rope_dim;
  const int DV = cfg.v_head_dim, R = cfg.kv_lora_rank, QD = DN + DR;
  if (!c.x.ensure(H * 4) || !c.q.ensure(static_cast<size_t>(NH) * QD * 4) || !c.ka.ensure((R + DR) * 4) ||
      !c.qabs.ensure(static_cast<size_t>(NH) * (R + DR) * 4) || !c.mix.ensure(static_cast<size_t>(NH) * R * 4) ||
      !c.ho.ensure(static_cast<size_t>(NH) * DV * 4) || !c.y.ensure(H * 4) || !c.rowf.ensure((R + DR) * 4)) {
    set_err("cudaMalloc of decode scratch failed");
    return -1;
  }
  const size_t io = static_cast<size_t>(2 * H + (R + DR) + 64) * 4 + R + 16;
  if (!c.pin_io.ensure(io)) {
    set_err("cudaMallocHost failed");
    return -1;
  }
  float *px = c.pin_io.as<float>();
  float *py = px + H;
  float *prow = py + H;
  uint32_t *perr = reinterpret_cast<uint32_t *>(prow + R + DR);
  int8_t *pq8 = reinterpret_cast<int8_t *>(perr + 16);
  memcpy(px, x, H * sizeof(float));
  CK(cudaMemcpyAsync(c.x.p, px, H * 4, cudaMemcpyHostToDevice, c.stream));
  CK(gemv_bf16(c.q.as<float>(), c.x.as<float>(), W.q, H, NH * QD, 1, c.stream));
  CK(gemv_bf16(c.ka.as<float>(), c.x.as<float>(), W.kva, H, R + DR, 1, c.stream, true));
  if (ds.fmt == FMT_BF16) {
    CK(append_bf16(ds.kv, 0, c.ka.as<float>(), W.kvan, 1, R, DR, position, cfg.rms_eps, cfg.rope_theta,
                   c.rowf.as<float>(), c.stream));
    if (ds.kvf)
      CK(cudaMemcpyAsync(ds.kvf + static_cast<size_t>(position) * (R + DR), c.rowf.p, (R + DR) * sizeof(float),
                         cudaMemcpyDeviceToDevice, c.stream));
  } else
    CK(append_q8(ds.lat8, ds.lscale, ds.rope16, 0, c.ka.as<float>(), W.kvan, 1, R, DR, position, cfg.rms_eps,
                 cfg.rope_theta, c.stream));
  // the plan's upload goes before the absorb kernel, so that the attend follows
  // it directly and may start while it runs (the rows are complete by then)
  if (plan_state(c, ds, position + 1, NH) != 0) return -1;
  CK(absorb(c.qabs.as<float>(), c.q.as<float>(), W.kvb, 1, NH, DN, DV, DR, R, position, cfg.rope_theta, c.stream));
  if (attend_state(c, ds, NH, 1.0f / sqrtf(static_cast<float>(QD)), true) != 0) return -1;
  CK(vup(c.ho.as<float>(), c.mix.as<float>(), W.kvb, 1, NH, DN, DV, R, c.stream));
  CK(gemv_bf16(c.y.as<float>(), c.ho.as<float>(), W.o, NH * DV, H, 1, c.stream));
  CK(cudaMemcpyAsync(py, c.y.p, H * 4, cudaMemcpyDeviceToHost, c.stream));
  CK(cudaMemcpyAsync(perr, c.plan.err_word(), 4, cudaMemcpyDeviceToHost, c.stream));
  if (ds.fmt == FMT_BF16) {
    CK(cudaMemcpyAsync(prow, c.rowf.p, (R + DR) * 4, cudaMemcpyDeviceToHost, c.stream));
  } else {
    const size_t pos = position;
    CK(cudaMemcpyAsync(pq8, ds.lat8 + pos * R, R, cudaMemcpyDeviceToHost, c.stream));
    CK(cudaMemcpyAsync(prow, ds.lscale + pos, 4, cudaMemcpyDeviceToHost, c.stream));
    CK(cudaMemcpyAsync(prow + 1, ds.rope16 + pos * DR, DR * 2, cudaMemcpyDeviceToHost, c.stream));
  }
  CK(cudaStreamSynchronize(c.stream));
  if (*perr != 0) {
    set_err("attend kernel reported device error 0x%x", *perr);
    return -1;
  }
  memcpy(out, py, H * sizeof(float));
  if (ds.fmt == FMT_BF16) {
    memcpy(mir_lat, prow, R * sizeof(float));
    memcpy(mir_rope, prow + R, DR * sizeof(float));
  } else {
    memcpy(mir_q8, pq8, R);
    memcpy(mir_scale, prow, 4);
    memcpy(mir_rope16, prow + 1, DR * 2);
  }
  return 0;
}

// `count` consecutive tokens of one bf16 state in one pass: projections,
// appends of rows [position, position + count), attends (token t over rows
// [0, position + t], each cut exactly as its own decode cuts it), V up and
// o_proj.  Every kernel computes each token as decode_one does, so the outputs
// and rows equal `count` serial decodes bit for bit.
int decode_block(Ctx &c, DevState &ds, const KvlMlaConfig &cfg, const DevW &W, const float *x, float *out,
                 int position, int count, float *mir_lat, float *mir_rope) {
  const int H = cfg.hidden_size, NH = cfg.num_heads, DN = cfg.qk_nope_dim, DR = cfg.qk_rope_dim;
  const int DV = cfg.v_head_dim, R = cfg.kv_lora_rank, QD = DN + DR;
  const size_t n = count;
  if (!c.x.ensure(n * H * 4) || !c.q.ensure(n * NH * QD * 4) || !c.ka.ensure(n * (R + DR) * 4) ||
      !c.qabs.ensure(n * NH * (R + DR) * 4) || !c.mix.ensure(n * NH * R * 4) || !c.ho.ensure(n * NH * DV * 4) ||
      !c.y.ensure(n * H * 4) || !c.rowf.ensure(n * (R + DR) * 4)) {
    set_err("cudaMalloc of decode scratch failed");
    return -1;
  }
  std::vector<int> lens(count);
  std::vector<long long> row0(count, 0);
  for (int t = 0; t < count; ++t) lens[t] = position + t + 1;
  HostPlan hp;
  if (build_concat_plan(hp, count, lens.data(), row0.data(), c.sms) != 0) {
    set_err("block attend plan failed");
    return -1;
  }
  if (!c.pin_plan.ensure(64 * 1024) || c.plan.upload(hp, NH, R, c.stream, c.pin_plan.p, c.pin_plan.n) != 0) {
    set_err("attend plan upload failed");
    return -1;
  }
  CK(cudaMemcpyAsync(c.x.p, x, n * H * 4, cudaMemcpyHostToDevice, c.stream));
  CK(gemv_bf16(c.q.as<float>(), c.x.as<float>(), W.q, H, NH * QD, count, c.stream));
  CK(gemv_bf16(c.ka.as<float>(), c.x.as<float>(), W.kva, H, R + DR, count, c.stream, true));
  CK(append_bf16(ds.kv, 0, c.ka.as<float>(), W.kvan, count, R, DR, position, cfg.rms_eps, cfg.rope_theta,
                 c.rowf.as<float>(), c.stream));
  if (ds.kvf)
    CK(cudaMemcpyAsync(ds.kvf + static_cast<size_t>(position) * (R + DR), c.rowf.p, n * (R + DR) * sizeof(float),
                       cudaMemcpyDeviceToDevice, c.stream));
  CK(absorb(c.qabs.as<float>(), c.q.as<float>(), W.kvb, count, NH, DN, DV, DR, R, position, cfg.rope_theta,
            c.stream));
  AttendLaunch a;
  a.nh = NH;
  a.R = R;
  a.DR = DR;
  a.rows = ds.cap_pad;
  a.q = c.qabs.as<float>();
  a.out = c.mix.as<float>();
  a.kv = ds.kv;
  a.kvf = ds.kvf;
  a.softmax_scale = 1.0f / sqrtf(static_cast<float>(QD));
  if (c.plan.launch(a, c.stream) != 0) {
    set_err("attend launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  CK(vup(c.ho.as<float>(), c.mix.as<float>(), W.kvb, count, NH, DN, DV, R, c.stream));
  CK(gemv_bf16(c.y.as<float>(), c.ho.as<float>(), W.o, NH * DV, H, count, c.stream));
  uint32_t err = 0;
  CK(cudaMemcpyAsync(&err, c.plan.err_word(), 4, cudaMemcpyDeviceToHost, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  if (err != 0) {
    set_err("attend kernel reported device error 0x%x", err);
    return -1;
  }
  CK(cudaMemcpy(out, c.y.p, n * H * 4, cudaMemcpyDeviceToHost));
  std::vector<float> rows(n * (R + DR));
  CK(cudaMemcpy(rows.data(), c.rowf.p, rows.size() * 4, cudaMemcpyDeviceToHost));
  for (size_t t = 0; t < n; ++t) {
    memcpy(mir_lat + t * R, rows.data() + t * (R + DR), R * sizeof(float));
    memcpy(mir_rope + t * DR, rows.data() + t * (R + DR) + R, DR * sizeof(float));
  }
  return 0;
}

// kv_a projection + append of rows 0..S-1 (state prefill, both formats).
int prefill_state(Ctx &c, DevState &ds, const KvlMlaConfig &cfg, const DevW &W, const float *x, int S) {
  const int H = cfg.hidden_size, R = cfg.kv_lora_rank, DR = cfg.qk_rope_dim;
  if (!c.x.ensure(static_cast<size_t>(S) * H * 4) || !c.ka.ensure(static_cast<size_t>(S) * (R + DR) * 4) ||
      !c.rowf.ensure(static_cast<size_t>(S) * (R + DR) * 4)) {
    set_err("cudaMalloc of prefill scratch failed");
    return -1;
  }
  CK(cudaMemcpyAsync(c.x.p, x, static_cast<size_t>(S) * H * 4, cudaMemcpyHostToDevice, c.stream));
  CK(gemv_bf16(c.ka.as<float>(), c.x.as<float>(), W.kva, H, R + DR, S, c.stream, true));
  if (ds.fmt == FMT_BF16) {
    CK(append_bf16(ds.kv, 0, c.ka.as<float>(), W.kvan, S, R, DR, 0, cfg.rms_eps, cfg.rope_theta,
                   c.rowf.as<float>(), c.stream));
    if (ds.kvf)
      CK(cudaMemcpyAsync(ds.kvf, c.rowf.p, static_cast<size_t>(S) * (R + DR) * sizeof(float),
                         cudaMemcpyDeviceToDevice, c.stream));
  } else
    CK(append_q8(ds.lat8, ds.lscale, ds.rope16, 0, c.ka.as<float>(), W.kvan, S, R, DR, 0, cfg.rms_eps,
                 cfg.rope_theta, c.stream));
  return 0;
}

}  // namespace

// Failure message for kvl_mla_cuda_last_error() from the other translation units.
void set_error_text(const char *msg) { set_err("%s", msg); }

}  // namespace kvl

using namespace kvl;

// =================================================================== misc
KVL_EXPORT const char *kvl_mla_cuda_last_error(void) { return g_err.c_str(); }

KVL_EXPORT int kvl_mla_cuda_weight_cache(int enable) {
  const int prev = weight_cache_enabled() ? 1 : 0;
  g_weight_cache.store(enable ? 1 : 0);
  return prev;
}

KVL_EXPORT size_t kvl_mla_cuda_state_device_bytes(const void *state) {
  if (!state) return 0;
  // Both state structs start with (capacity, len, R, DR) followed by the first
  // host mirror pointer, which is the registry key.
  const KvlMlaCompressedState *s = static_cast<const KvlMlaCompressedState *>(state);
  DevState *ds = find_state(s->latent);
  return ds ? ds->bytes : 0;
}

// =================================================================== bf16 (fp32-mirrored) state
// Reference: src/mla_compressed_state.c:24-50.
KVL_EXPORT int kvl_mla_compressed_state_init(KvlMlaCompressedState *state, const KvlMlaConfig *cfg, int capacity) {
  if (!state || !cfg || capacity <= 0 || cfg->kv_lora_rank <= 0 || cfg->qk_rope_dim <= 0 ||
      (cfg->qk_rope_dim & 1))
    return -1;
  memset(state, 0, sizeof(*state));
  const int R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  state->latent = static_cast<float *>(calloc(static_cast<size_t>(capacity) * R, sizeof(float)));
  state->rope = static_cast<float *>(calloc(static_cast<size_t>(capacity) * DR, sizeof(float)));
  DevState *ds = new DevState();
  // The production shape keeps bf16 rows for the tensor-core attend; other
  // shapes (the reference's probes) keep fp32 rows as the reference does.
  const bool f32_rows = !(cfg->num_heads == kHeads && R == kLatent && DR == kRope);
  if (!state->latent || !state->rope || alloc_dev_state(*ds, FMT_BF16, capacity, R, DR, f32_rows) != 0) {
    ds->release();
    delete ds;
    free(state->latent);
    free(state->rope);
    memset(state, 0, sizeof(*state));
    return -1;
  }
  register_state(state->latent, ds);
  state->capacity = capacity;
  state->kv_lora_rank = R;
  state->qk_rope_dim = DR;
  return 0;
}

KVL_EXPORT void kvl_mla_compressed_state_reset(KvlMlaCompressedState *state) {
  if (state) state->len = 0;
}

KVL_EXPORT int kvl_mla_compressed_state_truncate(KvlMlaCompressedState *state, int new_len) {
  if (!state || new_len < 0 || new_len > state->len) return -1;
  state->len = new_len;
  return 0;
}

KVL_EXPORT void kvl_mla_compressed_state_free(KvlMlaCompressedState *state) {
  if (!state) return;
  if (state->latent) {
    DevState *ds = unregister_state(state->latent);
    if (ds) {
      ds->release();
      delete ds;
    }
  }
  free(state->latent);
  free(state->rope);
  memset(state, 0, sizeof(*state));
}

KVL_EXPORT size_t kvl_mla_compressed_state_bytes(const KvlMlaCompressedState *state) {
  if (!state || state->capacity <= 0) return 0;
  return sizeof(*state) + static_cast<size_t>(state->capacity) *
                              (static_cast<size_t>(state->kv_lora_rank) + state->qk_rope_dim) * sizeof(float);
}

// Reference: src/mla_compressed_state.c:52-84.
KVL_EXPORT int kvl_mla_compressed_state_prefill_bf16(const float *x, int seq_len, const KvlMlaConfig *cfg,
                                                     const KvlMlaBF16 *w, KvlMlaCompressedState *state) {
  if (!x || !cfg || !w || !state || !w->kv_a_proj || !w->kv_a_norm || seq_len <= 0 || state->len != 0 ||
      seq_len > state->capacity || state->kv_lora_rank != cfg->kv_lora_rank ||
      state->qk_rope_dim != cfg->qk_rope_dim)
    return -1;
  const int H = cfg->hidden_size, R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  if (H <= 0 || R <= 0 || DR <= 0 || (DR & 1) || cfg->rope_theta <= 0.0f) return -1;
  DevState *ds = find_state(state->latent);
  if (!ds || ds->fmt != FMT_BF16) {
    set_err("state was not created by kvl_mla_compressed_state_init");
    return -1;
  }
  Ctx *c = get_ctx(ds->device);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  if (cudaSetDevice(ds->device) != cudaSuccess) return -1;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, false) != 0) return -1;
  if (prefill_state(*c, *ds, *cfg, W, x, seq_len) != 0) return -1;
  const float *rf = c->rowf.as<float>();
  CK(cudaMemcpy2DAsync(state->latent, R * 4, rf, (R + DR) * 4, R * 4, seq_len, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaMemcpy2DAsync(state->rope, DR * 4, rf + R, (R + DR) * 4, DR * 4, seq_len, cudaMemcpyDeviceToHost,
                       c->stream));
  CK(cudaStreamSynchronize(c->stream));
  ds->dev_len = seq_len;
  state->len = seq_len;
  return 0;
}

// Reference: src/mla_compressed_state.c:86-161.
KVL_EXPORT int kvl_mla_decode_compressed_bf16(float *out, const float *x, int position, const KvlMlaConfig *cfg,
                                              const KvlMlaBF16 *w, KvlMlaCompressedState *state) {
  if (!out || !x || !cfg || !w || !state || !w->q_proj || !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj ||
      !w->o_proj || position != state->len || position < 0 || position >= state->capacity ||
      state->kv_lora_rank != cfg->kv_lora_rank || state->qk_rope_dim != cfg->qk_rope_dim)
    return -1;
  if (!cfg_dims_ok(*cfg)) return -1;
  DevState *ds = find_state(state->latent);
  if (!ds || ds->fmt != FMT_BF16) {
    set_err("state was not created by kvl_mla_compressed_state_init");
    return -1;
  }
  Ctx *c = get_ctx(ds->device);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  if (cudaSetDevice(ds->device) != cudaSuccess) return -1;
  if (sync_bf16_state(*c, *ds, *state) != 0) return -1;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, true) != 0) return -1;
  const size_t R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  if (decode_one(*c, *ds, *cfg, W, x, out, position, state->latent + position * R, state->rope + position * DR,
                 nullptr, nullptr, nullptr) != 0)
    return -1;
  ds->dev_len = position + 1;
  state->len = position + 1;
  return 0;
}

// Reference: src/mla_compressed_state.c:163-184 (serial steps; here one pass
// over the block whose results equal the serial steps exactly).
KVL_EXPORT int kvl_mla_decode_compressed_block_bf16(float *out, const float *x, int count, int start_position,
                                                    const KvlMlaConfig *cfg, const KvlMlaBF16 *w,
                                                    KvlMlaCompressedState *state) {
  if (!out || !x || !cfg || !w || !state || count <= 0 || start_position != state->len || start_position < 0 ||
      count > state->capacity - start_position)
    return -1;
  if (!w->q_proj || !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj || !w->o_proj ||
      state->kv_lora_rank != cfg->kv_lora_rank || state->qk_rope_dim != cfg->qk_rope_dim || !cfg_dims_ok(*cfg))
    return -1;
  DevState *ds = find_state(state->latent);
  if (!ds || ds->fmt != FMT_BF16) {
    set_err("state was not created by kvl_mla_compressed_state_init");
    return -1;
  }
  Ctx *c = get_ctx(ds->device);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  if (cudaSetDevice(ds->device) != cudaSuccess) return -1;
  if (sync_bf16_state(*c, *ds, *state) != 0) return -1;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, true) != 0) return -1;
  const size_t R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  if (decode_block(*c, *ds, *cfg, W, x, out, start_position, count, state->latent + start_position * R,
                   state->rope + start_position * DR) != 0)
    return -1;
  ds->dev_len = start_position + count;
  state->len = start_position + count;
  return 0;
}

// =================================================================== Q8 state
// Reference: src/mla_compressed_q8_state.c:63-109.
KVL_EXPORT int kvl_mla_compressed_q8_state_init(KvlMlaCompressedQ8State *state, const KvlMlaConfig *cfg,
                                                int capacity) {
  if (!state || !cfg || capacity <= 0 || cfg->kv_lora_rank <= 0 || cfg->qk_rope_dim <= 0 ||
      (cfg->qk_rope_dim & 1))
    return -1;
  memset(state, 0, sizeof(*state));
  const int R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  state->latent_q8 = static_cast<int8_t *>(calloc(static_cast<size_t>(capacity) * R, 1));
  state->latent_scale = static_cast<float *>(calloc(static_cast<size_t>(capacity), sizeof(float)));
  state->rope_bf16 = static_cast<uint16_t *>(calloc(static_cast<size_t>(capacity) * DR, sizeof(uint16_t)));
  DevState *ds = new DevState();
  if (!state->latent_q8 || !state->latent_scale || !state->rope_bf16 ||
      alloc_dev_state(*ds, FMT_Q8, capacity, R, DR) != 0) {
    ds->release();
    delete ds;
    free(state->latent_q8);
    free(state->latent_scale);
    free(state->rope_bf16);
    memset(state, 0, sizeof(*state));
    return -1;
  }
  register_state(state->latent_q8, ds);
  state->capacity = capacity;
  state->kv_lora_rank = R;
  state->qk_rope_dim = DR;
  return 0;
}

KVL_EXPORT void kvl_mla_compressed_q8_state_reset(KvlMlaCompressedQ8State *state) {
  if (state) state->len = 0;
}

KVL_EXPORT int kvl_mla_compressed_q8_state_truncate(KvlMlaCompressedQ8State *state, int new_len) {
  if (!state || new_len < 0 || new_len > state->len) return -1;
  state->len = new_len;
  return 0;
}

KVL_EXPORT void kvl_mla_compressed_q8_state_free(KvlMlaCompressedQ8State *state) {
  if (!state) return;
  if (state->latent_q8) {
    DevState *ds = unregister_state(state->latent_q8);
    if (ds) {
      ds->release();
      delete ds;
    }
  }
  free(state->latent_q8);
  free(state->latent_scale);
  free(state->rope_bf16);
  memset(state, 0, sizeof(*state));
}

KVL_EXPORT size_t kvl_mla_compressed_q8_state_bytes(const KvlMlaCompressedQ8State *state) {
  if (!state || state->capacity <= 0) return 0;
  return sizeof(*state) + static_cast<size_t>(state->capacity) *
                              (static_cast<size_t>(state->kv_lora_rank) * sizeof(int8_t) + sizeof(float) +
                               static_cast<size_t>(state->qk_rope_dim) * sizeof(uint16_t));
}

// Reference: src/mla_compressed_q8_state.c:129-159.
KVL_EXPORT int kvl_mla_compressed_q8_state_prefill_bf16(const float *x, int seq_len, const KvlMlaConfig *cfg,
                                                        const KvlMlaBF16 *w, KvlMlaCompressedQ8State *state) {
  if (!x || !cfg || !w || !state || !w->kv_a_proj || !w->kv_a_norm || seq_len <= 0 || state->len != 0 ||
      seq_len > state->capacity || state->kv_lora_rank != cfg->kv_lora_rank ||
      state->qk_rope_dim != cfg->qk_rope_dim)
    return -1;
  const int H = cfg->hidden_size, R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  if (H <= 0 || R <= 0 || DR <= 0 || (DR & 1) || cfg->rope_theta <= 0.0f) return -1;
  DevState *ds = find_state(state->latent_q8);
  if (!ds || ds->fmt != FMT_Q8) {
    set_err("state was not created by kvl_mla_compressed_q8_state_init");
    return -1;
  }
  Ctx *c = get_ctx(ds->device);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  if (cudaSetDevice(ds->device) != cudaSuccess) return -1;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, false) != 0) return -1;
  if (prefill_state(*c, *ds, *cfg, W, x, seq_len) != 0) return -1;
  const size_t S = seq_len;
  CK(cudaMemcpyAsync(state->latent_q8, ds->lat8, S * R, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaMemcpyAsync(state->latent_scale, ds->lscale, S * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaMemcpyAsync(state->rope_bf16, ds->rope16, S * DR * 2, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  ds->dev_len = seq_len;
  state->len = seq_len;
  return 0;
}

// Reference: src/mla_compressed_q8_state.c:161-255.
KVL_EXPORT int kvl_mla_decode_compressed_q8_bf16(float *out, const float *x, int position, const KvlMlaConfig *cfg,
                                                 const KvlMlaBF16 *w, KvlMlaCompressedQ8State *state) {
  if (!out || !x || !cfg || !w || !state || !w->q_proj || !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj ||
      !w->o_proj || position != state->len || position < 0 || position >= state->capacity ||
      state->kv_lora_rank != cfg->kv_lora_rank || state->qk_rope_dim != cfg->qk_rope_dim)
    return -1;
  if (!cfg_dims_ok(*cfg)) return -1;
  DevState *ds = find_state(state->latent_q8);
  if (!ds || ds->fmt != FMT_Q8) {
    set_err("state was not created by kvl_mla_compressed_q8_state_init");
    return -1;
  }
  Ctx *c = get_ctx(ds->device);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  if (cudaSetDevice(ds->device) != cudaSuccess) return -1;
  if (sync_q8_state(*c, *ds, *state) != 0) return -1;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, true) != 0) return -1;
  const size_t R = cfg->kv_lora_rank, DR = cfg->qk_rope_dim;
  if (decode_one(*c, *ds, *cfg, W, x, out, position, nullptr, nullptr, state->latent_q8 + position * R,
                 state->latent_scale + position, state->rope_bf16 + position * DR) != 0)
    return -1;
  ds->dev_len = position + 1;
  state->len = position + 1;
  return 0;
}

// =================================================================== prefill
// Production shape (16 heads, DN 128, DR 64, DV 128, R 512): tcgen05 GEMMs for
// the projections (RoPE of q fused into the q_proj epilogue), the latent pool
// by append_bf16, and the causal flash kernel in the non-absorbed form.  Other
// shapes (the reference probes' tiny ones) run the causal attention in the
// absorbed form through the decode attend kernel (query t attends [0, t]).
namespace kvl {
namespace {

bool fast_prefill_shape(const KvlMlaConfig &c) {
  return c.num_heads == 16 && c.qk_nope_dim == 128 && c.qk_rope_dim == 64 && c.v_head_dim == 128 &&
         c.kv_lora_rank == 512 && c.hidden_size % 8 == 0;
}

struct PrefillWs {
  size_t off[11];
  size_t total;
};

PrefillWs prefill_layout(const KvlMlaConfig &c, int S) {
  const size_t s = S, H = c.hidden_size, NH = c.num_heads, QD = c.qk_nope_dim + c.qk_rope_dim;
  const size_t R = c.kv_lora_rank, DR = c.qk_rope_dim, DV = c.v_head_dim, DN = c.qk_nope_dim;
  size_t sz[10];
  int n;
  if (fast_prefill_shape(c)) {
    // xf, xb, q (bf16, rope applied), kva (fp32), pool (bf16 latent|rope), kv (bf16), o (bf16), cos/sin, err,
    // the flash kernel's key-range pieces (partial O and log-sum-exp; context-parallel launches)
    const size_t f[10] = {s * H * 4, s * H * 2, s * NH * QD * 2, s * (R + DR) * 4, s * (R + DR) * 2,
                          s * NH * (DN + DV) * 2, s * NH * DV * 2, s * (DR / 2) * 8, 256,
                          static_cast<size_t>(kFlashMaxUnits) * 128 * (128 + 1) * 4};
    for (int i = 0; i < 10; ++i) sz[i] = f[i];
    n = 10;
  } else {
    // xf, q, kva, qabs, mix, head_out, pool (bf16), pool (fp32: what the
    // CUDA-core attend reads for shapes other than 16 x 512 x 64)
    const size_t f[8] = {s * H * 4, s * NH * QD * 4, s * (R + DR) * 4, s * NH * (R + DR) * 4, s * NH * R * 4,
                         s * NH * DV * 4, (s + kTileTok) * (R + DR) * 2, (s + kTileTok) * (R + DR) * 4};
    for (int i = 0; i < 8; ++i) sz[i] = f[i];
    n = 8;
  }
  PrefillWs w;
  size_t o = 0;
  for (int i = 0; i < n; ++i) {
    w.off[i] = o;
    o += (sz[i] + 255) & ~size_t(255);
  }
  for (int i = n; i < 11; ++i) w.off[i] = o;
  w.total = o;
  return w;
}

// Plans of the absorbed-form attend, cached per (device, S): query t covers rows [0, t].
std::mutex g_pplan_mu;
std::unordered_map<long long, DevicePlan *> g_pplan;

const DevicePlan *prefill_plan(int device, int S, int nh, int R, int sms) {
  const long long key = (static_cast<long long>(device) << 40) ^ (static_cast<long long>(nh) << 32) ^
                        (static_cast<long long>(R) << 20) ^ S;
  std::lock_guard<std::mutex> lk(g_pplan_mu);
  auto it = g_pplan.find(key);
  if (it != g_pplan.end()) return it->second;
  std::vector<int> lens(S);
  std::vector<long long> row0(S, 0);
  for (int t = 0; t < S; ++t) lens[t] = t + 1;
  HostPlan hp;
  if (build_attend_plan(hp, S, lens.data(), row0.data(), sms) != 0) return nullptr;
  DevicePlan *dp = new DevicePlan();
  if (dp->upload(hp, nh, R, nullptr, nullptr, 0) != 0 || cudaDeviceSynchronize() != cudaSuccess) {
    dp->release();
    delete dp;
    return nullptr;
  }
  g_pplan[key] = dp;
  return dp;
}

// Absorbed-form path; xf: fp32 tokens on the device.
int prefill_absorbed(int device, int sms, const KvlMlaConfig &cfg, const DevW &W, float *d_out, const float *xf,
                     int S, uint8_t *ws, const PrefillWs &L, cudaStream_t st) {
  const int H = cfg.hidden_size, NH = cfg.num_heads, DN = cfg.qk_nope_dim, DR = cfg.qk_rope_dim;
  const int DV = cfg.v_head_dim, R = cfg.kv_lora_rank, QD = DN + DR;
  float *q = reinterpret_cast<float *>(ws + L.off[1]);
  float *ka = reinterpret_cast<float *>(ws + L.off[2]);
  float *qabs = reinterpret_cast<float *>(ws + L.off[3]);
  float *mix = reinterpret_cast<float *>(ws + L.off[4]);
  float *ho = reinterpret_cast<float *>(ws + L.off[5]);
  uint16_t *pool = reinterpret_cast<uint16_t *>(ws + L.off[6]);
  float *poolf = reinterpret_cast<float *>(ws + L.off[7]);
  CK(gemv_bf16(q, xf, W.q, H, NH * QD, S, st));
  CK(gemv_bf16(ka, xf, W.kva, H, R + DR, S, st, true));
  CK(append_bf16(pool, 0, ka, W.kvan, S, R, DR, 0, cfg.rms_eps, cfg.rope_theta, poolf, st));
  CK(absorb(qabs, q, W.kvb, S, NH, DN, DV, DR, R, 0, cfg.rope_theta, st));
  const DevicePlan *dp = prefill_plan(device, S, NH, R, sms);
  if (!dp) {
    set_err("prefill attend plan failed");
    return -1;
  }
  AttendLaunch a;
  a.nh = NH;
  a.R = R;
  a.DR = DR;
  a.rows = static_cast<long long>(S) + kTileTok;
  a.q = qabs;
  a.out = mix;
  a.kv = pool;
  a.kvf = poolf;
  a.softmax_scale = 1.0f / sqrtf(static_cast<float>(QD));
  if (dp->launch(a, st) != 0) {
    set_err("prefill attend launch failed");
    return -1;
  }
  CK(vup(ho, mix, W.kvb, S, NH, DN, DV, R, st));
  CK(gemv_bf16(d_out, ho, W.o, NH * DV, H, S, st));
  return 0;
}

bool bf16_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  return make_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, inner, rows, row_bytes, 64, box_rows,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// Second stream of the prefill fork (per device): q_proj does not depend on
// the kv_a -> RMSNorm/RoPE -> kv_b chain, so the two run concurrently and
// each fills the SMs the other's last wave leaves idle.  `mu` keeps one
// fork/join's event records and waits together when threads share a device.
struct PrefillFork {
  cudaStream_t s2 = nullptr;
  cudaEvent_t fork = nullptr, rope = nullptr, qdone = nullptr;
  std::mutex mu;
};
std::mutex g_fork_mu;
std::unordered_map<int, PrefillFork *> g_fork;

PrefillFork *get_fork(int device) {
  std::lock_guard<std::mutex> lk(g_fork_mu);
  auto it = g_fork.find(device);
  if (it != g_fork.end()) return it->second;
  PrefillFork *f = new PrefillFork();
  if (cudaStreamCreateWithFlags(&f->s2, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&f->fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&f->rope, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&f->qdone, cudaEventDisableTiming) != cudaSuccess) {
    set_err("prefill: cannot create the second stream of device %d", device);
    delete f;
    return nullptr;
  }
  g_fork[device] = f;
  return f;
}

// tcgen05 path; xb: bf16 tokens on the device.  Returns -1 with a message.
// tcgen05 path over the query rows [r0, r1) of an S-row prompt (r0 % 128 == 0):
// projections, append and kv_b of those rows, attention of those queries over
// the keys [0, r1), o_proj into d_out rows [r0, r1).  xb: bf16 tokens on the
// device; the RoPE table and the error word are set up by the call with
// r0 == 0.  fork: run q_proj on a second stream beside the kv_a -> append ->
// kv_b chain (whole-prompt calls); chunked calls stay on `st`.  Returns -1
// with a message.
int prefill_fast(int sms, const KvlMlaConfig &cfg, const DevW &W, float *d_out, const uint16_t *xb, int S,
                 uint8_t *ws, const PrefillWs &L, cudaStream_t st, int r0 = 0, int r1 = -1, bool fork = true) {
  if (r1 < 0) r1 = S;
  const uint64_t H = cfg.hidden_size, s = S, m = static_cast<uint64_t>(r1 - r0), R0 = static_cast<uint64_t>(r0);
  const int M = r1 - r0;
  uint16_t *q = reinterpret_cast<uint16_t *>(ws + L.off[2]);
  float *kva = reinterpret_cast<float *>(ws + L.off[3]);
  uint16_t *pool = reinterpret_cast<uint16_t *>(ws + L.off[4]);
  uint16_t *kv = reinterpret_cast<uint16_t *>(ws + L.off[5]);
  uint16_t *o = reinterpret_cast<uint16_t *>(ws + L.off[6]);
  float2 *cs = reinterpret_cast<float2 *>(ws + L.off[7]);
  uint32_t *err = reinterpret_cast<uint32_t *>(ws + L.off[8]);
  if ((reinterpret_cast<uintptr_t>(xb) | reinterpret_cast<uintptr_t>(W.q) | reinterpret_cast<uintptr_t>(W.kva) |
       reinterpret_cast<uintptr_t>(W.kvb) | reinterpret_cast<uintptr_t>(W.o) | reinterpret_cast<uintptr_t>(W.kvan)) &
      15) {
    set_err("prefill: activations and weights must be 16-byte aligned");
    return -1;
  }
  if (r0 < 0 || r0 % 128 != 0 || r1 <= r0 || r1 > S) {
    set_err("prefill: invalid row range [%d, %d) of %d", r0, r1, S);
    return -1;
  }
  int dev = 0;
  CK(cudaGetDevice(&dev));
  PrefillFork *fk = get_fork(dev);
  if (!fk) return -1;
  std::lock_guard<std::mutex> lk(fk->mu);
  cudaStream_t sq = fork ? fk->s2 : st;
  if (r0 == 0) CK(cudaMemsetAsync(err, 0, 4, st));
  if (fork) {
    CK(cudaEventRecord(fk->fork, st));
    CK(cudaStreamWaitEvent(fk->s2, fk->fork, 0));
  }

  // Every kernel below is a programmatic dependent of the one before it on its
  // stream (each orders its global accesses after griddepcontrol.wait), so a
  // kernel's launch and set-up overlap the previous one's tail.
  // kva = x Wkva^T, fp32 [S][576], launched first: its 96 tiles (S = 4096) fill
  // 96 SMs for one round, and the q GEMM's CTA pairs take the idle SMs meanwhile.
  // When 3 tiles per 128 rows would leave more than half of the SMs idle (up to
  // 3072 rows on 148 SMs: a chunk of the host-buffer pipeline, a short prompt),
  // kv_a takes 64-column tiles, 9 per 128 rows (the same sums per element: the
  // MMA accumulates each element over K in the same order whatever the width).
  const int kva_bn = (M + 127) / 128 * 3 * 2 < sms ? 64 : 192;
  GemmParams g;
  memset(&g, 0, sizeof g);
  g.err = err;
  if (!bf16_map(&g.tm_a, xb + R0 * H, H, m, H * 2, 128) || !bf16_map(&g.tm_b, W.kva, H, 576, H * 2, kva_bn)) {
    set_err("prefill: tensor map (kv_a_proj)");
    return -1;
  }
  g.M = M;
  g.K = static_cast<int>(H);
  g.N = 576;
  g.c = kva + R0 * 576;
  g.ldc = 576;
  CK(launch_gemm(g, kva_bn, EPI_F32, sms, st, "gemm_kva", true));
  // q = x Wq^T with RoPE on each head's last 64 columns, bf16 [S][16][192]
  // (on the second stream when forked, after the RoPE table)
  GemmParams gq;
  memset(&gq, 0, sizeof gq);
  gq.err = err;
  if (!bf16_map(&gq.tm_a, xb + R0 * H, H, m, H * 2, 128) || !bf16_map(&gq.tm_b, W.q, H, 16 * 192, H * 2, 128)) {
    set_err("prefill: tensor map (q_proj)");
    return -1;
  }
  gq.M = M;
  gq.N = 16 * 192;
  gq.K = static_cast<int>(H);
  gq.c = q + R0 * 16 * 192;
  gq.ldc = 16 * 192;
  gq.rope_cs = cs + R0 * 32;
  if (r0 == 0) CK(launch_rope_table(cs, S, 64, cfg.rope_theta, sq));
  if (fork) CK(cudaEventRecord(fk->rope, sq));
  CK(launch_gemm_pair(gq, 256, EPI_QROPE, sms, sq, "gemm_q", true));
  if (fork) CK(cudaEventRecord(fk->qdone, sq));

  // latent = rmsnorm(kva[:512]) * kv_a_norm, k_rope = rope(kva[512:]) -> pool [S][576] bf16
  if (fork) CK(cudaStreamWaitEvent(st, fk->rope, 0));
  CK(append_rows_bf16(pool + R0 * 576, kva + R0 * 576, W.kvan, cs + R0 * 32, M, cfg.rms_eps, st));
  // kv = latent Wkvb^T, bf16 [S][16][256]
  if (!bf16_map(&g.tm_a, pool + R0 * 576, 512, m, 576 * 2, 128) ||
      !bf16_map(&g.tm_b, W.kvb, 512, 4096, 512 * 2, 128)) {
    set_err("prefill: tensor map (kv_b_proj)");
    return -1;
  }
  g.N = 4096;
  g.K = 512;
  g.c = kv + R0 * 4096;
  g.ldc = 4096;
  CK(launch_gemm_pair(g, 256, EPI_BF16, sms, st, "gemm_kvb", true));
  if (fork) CK(cudaStreamWaitEvent(st, fk->qdone, 0));  // join the second stream
  // causal attention of the queries [r0, r1) over the keys [0, r1) -> o bf16 [S][16][128]
  FlashParams f;
  memset(&f, 0, sizeof f);
  {
    const uint64_t qd[3] = {192, 16, s}, qs[2] = {192 * 2, 16 * 192 * 2};
    const uint64_t kd[3] = {256, 16, s}, ks[2] = {256 * 2, 16 * 256 * 2};
    const uint32_t box[3] = {64, 1, 128};
    if (!make_tmap_3d(&f.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, qd, qs, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_3d(&f.tm_kv, kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kd, ks, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !bf16_map(&f.tm_kr, pool, 576, s, 576 * 2, 128)) {
      set_err("prefill: tensor map (attention)");
      return -1;
    }
  }
  f.kr_col = 512;
  f.S = r1;
  f.q_tile0 = r0 / 128;
  f.scale_log2 = (1.0f / sqrtf(192.0f)) * 1.4426950408889634f;
  f.out = reinterpret_cast<__nv_bfloat16 *>(o);
  f.err = err;
  CK(launch_flash_prefill(f, sms, st, true));
  // out = o Wo^T, fp32 [S][H]
  // (CTA-pair GEMM: 256 x 256 tiles, each CTA of a pair loads 128 rows of Wo)
  if (!bf16_map(&g.tm_a, o + R0 * 2048, 2048, m, 2048 * 2, 128) ||
      !bf16_map(&g.tm_b, W.o, 2048, H, 2048 * 2, 128)) {
    set_err("prefill: tensor map (o_proj)");
    return -1;
  }
  g.N = static_cast<int>(H);
  g.K = 2048;
  g.c = d_out + R0 * H;
  g.ldc = static_cast<int>(H);
  g.rope_cs = nullptr;
  CK(launch_gemm_pair(g, 256, EPI_F32, sms, st, "gemm_o", true));
  return 0;
}

// ------------------------------------------------------------------ context-parallel prefill
// One prompt of S rows over `world` GPUs: 2 * world chunks of c = S / (2 world)
// rows; rank r owns chunk r (early keys) and chunk 2 world - 1 - r (late keys),
// so every rank has the same causal attention work.  The only exchange is the
// compressed 576-wide row of every token (latent | rotated k_rope, what the
// reference's streaming prefill appends per token, src/mla_prefill_streaming.c:
// 131-138): each rank projects and appends its own rows, the ranks all-gather
// them (S x 1152 bytes in all), and each rank expands K/V with kv_b for the keys
// its chunks see.  q_proj and o_proj stay with the rows' owner.
struct CpChunks {
  int c = 0;         // rows per chunk
  int a0 = 0, b0 = 0;  // first rows of the rank's two chunks
};

bool cp_chunks(int S, int rank, int world, CpChunks &k) {
  if (world <= 0 || rank < 0 || rank >= world || S <= 0 || S % (2 * world) != 0) return false;
  k.c = S / (2 * world);
  if (k.c % 128 != 0) return false;
  k.a0 = rank * k.c;
  k.b0 = (2 * world - 1 - rank) * k.c;
  return true;
}

// Projections of the rank's 2c rows, held compact (early chunk, then late
// chunk): the RoPE table of their positions; kv_a, RMSNorm and RoPE into d_send
// [2c][576] bf16; q_proj with RoPE into the workspace q [2c][16][192].  q_proj
// runs on the second stream beside the kv_a -> append chain.
int cp_project(int sms, const KvlMlaConfig &cfg, const DevW &W, const uint16_t *xb, int world, const CpChunks &k,
               uint16_t *d_send, uint8_t *ws, const PrefillWs &L, cudaStream_t st, PrefillFork *fk) {
  const int M = 2 * k.c;
  const uint64_t H = cfg.hidden_size, m = static_cast<uint64_t>(M);
  uint16_t *q = reinterpret_cast<uint16_t *>(ws + L.off[2]);
  float *kva = reinterpret_cast<float *>(ws + L.off[3]);
  float2 *cs = reinterpret_cast<float2 *>(ws + L.off[7]);
  uint32_t *err = reinterpret_cast<uint32_t *>(ws + L.off[8]);
  CK(cudaMemsetAsync(err, 0, 4, st));
  CK(cudaEventRecord(fk->fork, st));
  CK(cudaStreamWaitEvent(fk->s2, fk->fork, 0));
  const int kva_bn = (M + 127) / 128 * 3 * 2 < sms ? 64 : 192;
  // kv_a over a few hundred rows fills a fraction of the SMs: split its K range
  // (at most `world` parts of 2c rows fit the kva slot) and sum in the append
  const int tiles_mn = (M / 128) * (576 / kva_bn), ksteps = static_cast<int>((H + 63) / 64);
  int ks = 1;
  if (2 * tiles_mn <= sms)
    for (int want = std::min(world, sms / tiles_mn); want > 1 && ks == 1; --want)
      if (ksteps % want == 0) ks = want;
  GemmParams g;
  memset(&g, 0, sizeof g);
  g.err = err;
  if (!bf16_map(&g.tm_a, xb, H, m, H * 2, 128) || !bf16_map(&g.tm_b, W.kva, H, 576, H * 2, kva_bn)) {
    set_err("prefill (context parallel): tensor map (kv_a_proj)");
    return -1;
  }
  g.M = M;
  g.K = static_cast<int>(H);
  g.N = 576;
  g.c = kva;
  g.ldc = 576;
  g.ksplit = ks;
  g.c_bstride = static_cast<long long>(M) * 576;
  CK(launch_gemm(g, kva_bn, EPI_F32, sms, st, "gemm_kva"));
  // q_proj: CTA-pair tiles with RoPE in the epilogue, or, when those fill a
  // fraction of the SMs, a K split over 1-SM 192-wide tiles whose fp32
  // partials (in the x slot, unused by this form) are summed with the RoPE
  const int q_tiles = (M / 128) * (16 * 192 / 192);
  int qks = 1;
  if (2 * q_tiles <= sms)
    for (int want = sms / q_tiles; want > 1 && qks == 1; --want)
      if (ksteps % want == 0 && static_cast<size_t>(want) * M * 16 * 192 <= static_cast<size_t>(k.c) * 2 * world * H)
        qks = want;
  GemmParams gq;
  memset(&gq, 0, sizeof gq);
  gq.err = err;
  if (!bf16_map(&gq.tm_a, xb, H, m, H * 2, 128) ||
      !bf16_map(&gq.tm_b, W.q, H, 16 * 192, H * 2, qks > 1 ? 192 : 128)) {
    set_err("prefill (context parallel): tensor map (q_proj)");
    return -1;
  }
  gq.M = M;
  gq.N = 16 * 192;
  gq.K = static_cast<int>(H);
  gq.ldc = 16 * 192;
  CK(launch_rope_table_rows(cs, M, 64, cfg.rope_theta, k.c, k.a0, k.b0, fk->s2));
  CK(cudaEventRecord(fk->rope, fk->s2));
  if (qks > 1) {
    float *parts = reinterpret_cast<float *>(ws + L.off[0]);
    gq.c = parts;
    gq.ksplit = qks;
    gq.c_bstride = static_cast<long long>(M) * 16 * 192;
    CK(launch_gemm(gq, 192, EPI_F32, sms, fk->s2, "gemm_q"));
    CK(sum_parts_qrope(q, parts, qks, gq.c_bstride, cs, M, fk->s2));
  } else {
    gq.c = q;
    gq.rope_cs = cs;
    CK(launch_gemm_pair(gq, 256, EPI_QROPE, sms, fk->s2, "gemm_q"));
  }
  CK(cudaEventRecord(fk->qdone, fk->s2));
  CK(cudaStreamWaitEvent(st, fk->rope, 0));
  CK(append_rows_bf16(d_send, kva, W.kvan, cs, M, cfg.rms_eps, st, ks, g.c_bstride));
  CK(cudaStreamWaitEvent(st, fk->qdone, 0));
  return 0;
}

// K/V expanded with kv_b from the gathered rows for the keys the rank's chunks
// see ([0, end of its late chunk), read through the zigzag tile map), the causal attention
// of both chunks in one flash launch (the late chunk as the kernel's main query
// range, the early one as its second range, queries and output compact), and
// o_proj of the 2c rows into d_out [2c][H] fp32.
int cp_attend(int sms, const KvlMlaConfig &cfg, const DevW &W, float *d_out, const uint16_t *d_recv, int world,
              const CpChunks &k, uint8_t *ws, const PrefillWs &L, cudaStream_t st) {
  const int kmax = k.b0 + k.c, M = 2 * k.c;
  const uint64_t H = cfg.hidden_size, s = static_cast<uint64_t>(kmax), m = static_cast<uint64_t>(M);
  uint16_t *q = reinterpret_cast<uint16_t *>(ws + L.off[2]);
  uint16_t *kv = reinterpret_cast<uint16_t *>(ws + L.off[5]);
  uint16_t *o = reinterpret_cast<uint16_t *>(ws + L.off[6]);
  uint32_t *err = reinterpret_cast<uint32_t *>(ws + L.off[8]);
  // the gathered rows are read in place, in prompt order through the zigzag
  // tile map (kv_b's A rows and the flash kernel's k_rope rows)
  const uint64_t S_all = static_cast<uint64_t>(2 * world) * k.c;
  // kv = latent Wkvb^T for the keys [0, kmax), bf16 [kmax][16][256]
  GemmParams g;
  memset(&g, 0, sizeof g);
  g.err = err;
  if (!bf16_map(&g.tm_a, d_recv, 512, S_all, 576 * 2, 128) || !bf16_map(&g.tm_b, W.kvb, 512, 4096, 512 * 2, 128)) {
    set_err("prefill (context parallel): tensor map (kv_b_proj)");
    return -1;
  }
  g.M = kmax;
  g.N = 4096;
  g.K = 512;
  g.c = kv;
  g.ldc = 4096;
  g.zz_world = world;
  g.zz_c128 = k.c / 128;
  CK(launch_gemm_pair(g, 256, EPI_BF16, sms, st, "gemm_kvb"));
  FlashParams f;
  memset(&f, 0, sizeof f);
  {
    const uint64_t qd[3] = {192, 16, m}, qs[2] = {192 * 2, 16 * 192 * 2};
    const uint64_t kd[3] = {256, 16, s}, ks[2] = {256 * 2, 16 * 256 * 2};
    const uint32_t box[3] = {64, 1, 128};
    if (!make_tmap_3d(&f.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, qd, qs, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_3d(&f.tm_kv, kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kd, ks, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !bf16_map(&f.tm_kr, d_recv, 576, S_all, 576 * 2, 128)) {
      set_err("prefill (context parallel): tensor map (attention)");
      return -1;
    }
  }
  f.kr_col = 512;
  f.S = kmax;
  f.q_tile0 = k.b0 / 128;
  f.lo_t0 = k.a0 / 128;
  f.lo_t1 = (k.a0 + k.c) / 128;
  f.q_compact = 1;
  f.scale_log2 = (1.0f / sqrtf(192.0f)) * 1.4426950408889634f;
  f.out = reinterpret_cast<__nv_bfloat16 *>(o);
  f.err = err;
  // few items per rank at larger worlds: the launcher cuts the long ones by key range
  f.kpiece = -1;
  f.part_o = reinterpret_cast<float *>(ws + L.off[9]);
  f.part_lse = f.part_o + static_cast<size_t>(kFlashMaxUnits) * 128 * 128;
  f.zz_world = world;
  f.zz_c128 = k.c / 128;
  CK(launch_flash_prefill(f, sms, st));
  // out = o Wo^T, fp32 [2c][H].  At a few hundred rows the CTA-pair tiles
  // would fill a fraction of the SMs, so the K range is split over 1-SM tiles
  // (fp32 partials in the x slot, which this form does not use: at most
  // `world` parts of 2c rows) and the partials summed.
  const int tiles_mn = (M / 128) * static_cast<int>((H + 255) / 256);
  int ks = 1;
  if (2 * tiles_mn <= sms)
    for (int want = std::min(world, sms / tiles_mn); want > 1 && ks == 1; --want)
      if ((2048 / 64) % want == 0) ks = want;
  if (ks > 1) {
    float *parts = reinterpret_cast<float *>(ws + L.off[0]);
    if (!bf16_map(&g.tm_a, o, 2048, m, 2048 * 2, 128) || !bf16_map(&g.tm_b, W.o, 2048, H, 2048 * 2, 256)) {
      set_err("prefill (context parallel): tensor map (o_proj)");
      return -1;
    }
    g.M = M;
    g.N = static_cast<int>(H);
    g.K = 2048;
    g.c = parts;
    g.ldc = static_cast<int>(H);
    g.ksplit = ks;
    g.c_bstride = static_cast<long long>(M) * static_cast<long long>(H);
    CK(launch_gemm(g, 256, EPI_F32, sms, st, "gemm_o"));
    CK(sum_parts(d_out, parts, ks, g.c_bstride, g.c_bstride, st));
    return 0;
  }
  if (!bf16_map(&g.tm_a, o, 2048, m, 2048 * 2, 128) || !bf16_map(&g.tm_b, W.o, 2048, H, 2048 * 2, 128)) {
    set_err("prefill (context parallel): tensor map (o_proj)");
    return -1;
  }
  g.M = M;
  g.N = static_cast<int>(H);
  g.K = 2048;
  g.c = d_out;
  g.ldc = static_cast<int>(H);
  CK(launch_gemm_pair(g, 256, EPI_F32, sms, st, "gemm_o"));
  return 0;
}

}  // namespace
}  // namespace kvl

// Row boundaries of the host-buffer prefill pipeline: equal chunks of a
// multiple of 128 rows; returns the chunk count, bounds[0..count] the
// boundaries.  Measured at S = 4096 on one B200 (PCIe about 52 GB/s each way
// alone, ~40 GB/s each way when both directions run; a 1024-row chunk computes
// in ~140 us, mostly one round of each GEMM): 3 chunks 1.14 ms per call,
// 4 chunks 1.01 ms, 4 chunks without the second stream or with 192-column kv_a
// tiles 1.02-1.04 ms, 5 chunks with half-size end chunks 1.06-1.08 ms,
// 8 chunks 1.32 ms -- smaller chunks overlap more copy time, but every chunk
// pays the latency of its seven kernels.  Replaying each chunk as a recorded
// CUDA graph was slower (1.09 ms).
static int prefill_chunk_bounds(int seq_len, int *bounds) {
  const int nch = seq_len >= 2048 ? 4 : seq_len >= 1024 ? 2 : 1;
  const int rows = ((seq_len + nch - 1) / nch + 127) / 128 * 128;
  int n = 0;
  bounds[0] = 0;
  for (int r0 = 0; r0 < seq_len; r0 += rows) bounds[++n] = std::min(seq_len, r0 + rows);
  return n;
}

// Reference: src/mla_prefill_streaming.c:78-206 (validation :80-85).
KVL_EXPORT int kvl_mla_prefill_bf16(float *out, const float *x, int seq_len, const KvlMlaConfig *cfg,
                                    const KvlMlaBF16 *w) {
  if (!out || !x || !cfg || !w || !w->q_proj || !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj || !w->o_proj ||
      seq_len <= 0 || cfg->hidden_size <= 0 || cfg->num_heads <= 0 || cfg->qk_nope_dim <= 0 ||
      cfg->qk_rope_dim <= 0 || (cfg->qk_rope_dim & 1) || cfg->v_head_dim <= 0 || cfg->kv_lora_rank <= 0 ||
      cfg->rope_theta <= 0.0f)
    return -1;
  const int dev = current_device();
  if (dev < 0) return -1;
  Ctx *c = get_ctx(dev);
  if (!c) return -1;
  std::lock_guard<std::mutex> lk(c->mu);
  const size_t s = seq_len, H = cfg->hidden_size;
  DevW W;
  if (stage_weights(*c, *cfg, *w, W, true) != 0) return -1;
  const PrefillWs L = prefill_layout(*cfg, seq_len);
  if (!c->kvtmp.ensure(L.total) || !c->y.ensure(s * H * 4)) {
    set_err("cudaMalloc of prefill scratch failed");
    return -1;
  }
  uint8_t *ws = c->kvtmp.as<uint8_t>();
  float *xf = reinterpret_cast<float *>(ws + L.off[0]);
  int bounds[kMaxPrefillChunks + 1];
  const int nch = fast_prefill_shape(*cfg) ? prefill_chunk_bounds(seq_len, bounds) : 1;
  if (nch > 1) {
    // Chunked pipeline: the H2D copy of chunk i+1 and the D2H copy of chunk
    // i-1 run on their own streams while chunk i computes (its queries attend
    // the keys of every chunk before it, which are already on the device).
    if (!c->copy_in) {
      if (cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking) != cudaSuccess ||
          cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking) != cudaSuccess) {
        set_err("prefill: cannot create copy streams");
        return -1;
      }
      for (int i = 0; i < kMaxPrefillChunks; ++i)
        if (cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_out[i], cudaEventDisableTiming) != cudaSuccess) {
          set_err("prefill: cannot create copy events");
          return -1;
        }
    }
    uint16_t *xb = reinterpret_cast<uint16_t *>(ws + L.off[1]);
    float *y = c->y.as<float>();
    // the weights were staged on c->stream: the copies and kernels below follow it
    CK(cudaEventRecord(c->ev_out[0], c->stream));
    CK(cudaStreamWaitEvent(c->copy_in, c->ev_out[0], 0));
    for (int i = 0; i < nch; ++i) {
      const size_t off = static_cast<size_t>(bounds[i]) * H, n = static_cast<size_t>(bounds[i + 1] - bounds[i]) * H;
      CK(cudaMemcpyAsync(xf + off, x + off, n * 4, cudaMemcpyHostToDevice, c->copy_in));
      CK(cudaEventRecord(c->ev_in[i], c->copy_in));
    }
    for (int i = 0; i < nch; ++i) {
      const int r0 = bounds[i], r1 = bounds[i + 1];
      const size_t off = static_cast<size_t>(r0) * H, n = static_cast<size_t>(r1 - r0) * H;
      CK(cudaStreamWaitEvent(c->stream, c->ev_in[i], 0));
      CK(f32_to_bf16(xb + off, xf + off, static_cast<long long>(n), c->stream));
      // q_proj on the second stream beside the kv_a -> append -> kv_b chain
      if (prefill_fast(c->sms, *cfg, W, y, xb, seq_len, ws, L, c->stream, r0, r1, true) != 0) return -1;
      CK(cudaEventRecord(c->ev_out[i], c->stream));
      CK(cudaStreamWaitEvent(c->copy_out, c->ev_out[i], 0));
      CK(cudaMemcpyAsync(out + off, y + off, n * 4, cudaMemcpyDeviceToHost, c->copy_out));
    }
    uint32_t err = 0;
    CK(cudaMemcpyAsync(&err, ws + L.off[8], 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaStreamSynchronize(c->copy_out));
    if (err != 0) {
      set_err("prefill kernel reported device error 0x%x", err);
      return -1;
    }
    return 0;
  }
  CK(cudaMemcpyAsync(xf, x, s * H * 4, cudaMemcpyHostToDevice, c->stream));
  int rc;
  if (fast_prefill_shape(*cfg)) {
    uint16_t *xb = reinterpret_cast<uint16_t *>(ws + L.off[1]);
    CK(f32_to_bf16(xb, xf, static_cast<long long>(s * H), c->stream));
    rc = prefill_fast(c->sms, *cfg, W, c->y.as<float>(), xb, seq_len, ws, L, c->stream);
  } else {
    rc = prefill_absorbed(dev, c->sms, *cfg, W, c->y.as<float>(), xf, seq_len, ws, L, c->stream);
  }
  if (rc != 0) return -1;
  CK(cudaMemcpyAsync(out, c->y.p, s * H * 4, cudaMemcpyDeviceToHost, c->stream));
  uint32_t err = 0;
  if (fast_prefill_shape(*cfg))
    CK(cudaMemcpyAsync(&err, ws + L.off[8], 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  if (err != 0) {
    set_err("prefill kernel reported device error 0x%x", err);
    return -1;
  }
  return 0;
}

KVL_EXPORT size_t kvl_mla_prefill_workspace_bytes(const KvlMlaConfig *cfg, int seq_len) {
  if (!cfg || seq_len <= 0 || !cfg_dims_ok(*cfg)) return 0;
  return prefill_layout(*cfg, seq_len).total;
}

KVL_EXPORT int kvl_mla_prefill_dev(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, float *d_out,
                                   const uint16_t *d_x, int seq_len, void *d_workspace, size_t workspace_bytes,
                                   void *stream) {
  if (!cfg || !w || !d_out || !d_x || seq_len <= 0 || !d_workspace || !cfg_dims_ok(*cfg) || !w->q_proj ||
      !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj || !w->o_proj) {
    set_err("invalid prefill arguments");
    return -1;
  }
  const PrefillWs L = prefill_layout(*cfg, seq_len);
  if (workspace_bytes < L.total) {
    set_err("prefill workspace too small (%zu < %zu)", workspace_bytes, L.total);
    return -1;
  }
  if (reinterpret_cast<uintptr_t>(d_workspace) & 255) {
    set_err("prefill workspace must be 256-byte aligned");
    return -1;
  }
  const int dev = current_device();
  if (dev < 0) return -1;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(d_workspace);
  DevW W{w->q_proj, w->kv_a_proj, w->kv_a_norm, w->kv_b_proj, w->o_proj};
  if (fast_prefill_shape(*cfg)) return prefill_fast(sms, *cfg, W, d_out, d_x, seq_len, ws, L, st);
  float *xf = reinterpret_cast<float *>(ws + L.off[0]);
  CK(bf16_to_f32(xf, d_x, static_cast<long long>(seq_len) * cfg->hidden_size, st));
  return prefill_absorbed(dev, sms, *cfg, W, d_out, xf, seq_len, ws, L, st);
}

// Checks shared by the two context-parallel calls; fills L, sms, the chunks.
static int cp_setup(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, int seq_len, int rank, int world,
                    void *d_workspace, size_t workspace_bytes, PrefillWs &L, int &sms, CpChunks &k) {
  if (!cfg || !w || seq_len <= 0 || !d_workspace || !cfg_dims_ok(*cfg) || !fast_prefill_shape(*cfg) ||
      !w->q_proj || !w->kv_a_proj || !w->kv_a_norm || !w->kv_b_proj || !w->o_proj) {
    set_err("invalid context-parallel prefill arguments (production head shape required)");
    return -1;
  }
  if (!cp_chunks(seq_len, rank, world, k)) {
    set_err("context-parallel prefill: seq_len %d must split into %d chunks of a multiple of 128 rows "
            "(rank %d of %d)", seq_len, 2 * world, rank, world);
    return -1;
  }
  L = prefill_layout(*cfg, seq_len);
  if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(d_workspace) & 255)) {
    set_err("context-parallel prefill: workspace too small or not 256-byte aligned (%zu < %zu)", workspace_bytes,
            L.total);
    return -1;
  }
  const int dev = current_device();
  if (dev < 0) return -1;
  sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return 0;
}

KVL_EXPORT int kvl_mla_prefill_cp_begin(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, const uint16_t *d_x,
                                        int seq_len, int rank, int world, uint16_t *d_send, void *d_workspace,
                                        size_t workspace_bytes, void *stream) {
  PrefillWs L;
  int sms = 0;
  CpChunks k;
  if (cp_setup(cfg, w, seq_len, rank, world, d_workspace, workspace_bytes, L, sms, k) != 0) return -1;
  if (!d_x || !d_send || ((reinterpret_cast<uintptr_t>(d_x) | reinterpret_cast<uintptr_t>(d_send)) & 15)) {
    set_err("context-parallel prefill: d_x and d_send must be 16-byte aligned device pointers");
    return -1;
  }
  DevW W{w->q_proj, w->kv_a_proj, w->kv_a_norm, w->kv_b_proj, w->o_proj};
  PrefillFork *fk = get_fork(current_device());
  if (!fk) return -1;
  std::lock_guard<std::mutex> lk(fk->mu);
  return cp_project(sms, *cfg, W, d_x, world, k, d_send, static_cast<uint8_t *>(d_workspace), L,
                    static_cast<cudaStream_t>(stream), fk);
}

KVL_EXPORT int kvl_mla_prefill_cp_end(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, float *d_out,
                                      int seq_len, int rank, int world, const uint16_t *d_recv, void *d_workspace,
                                      size_t workspace_bytes, void *stream) {
  PrefillWs L;
  int sms = 0;
  CpChunks k;
  if (cp_setup(cfg, w, seq_len, rank, world, d_workspace, workspace_bytes, L, sms, k) != 0) return -1;
  if (!d_out || !d_recv || ((reinterpret_cast<uintptr_t>(d_out) | reinterpret_cast<uintptr_t>(d_recv)) & 15)) {
    set_err("context-parallel prefill: d_out and d_recv must be 16-byte aligned device pointers");
    return -1;
  }
  DevW W{w->q_proj, w->kv_a_proj, w->kv_a_norm, w->kv_b_proj, w->o_proj};
  return cp_attend(sms, *cfg, W, d_out, d_recv, world, k, static_cast<uint8_t *>(d_workspace), L,
                   static_cast<cudaStream_t>(stream));
}

// =================================================================== attend plans
struct KvlMlaAttendPlan {
  int device = 0;
  int nh = 0, R = 0;
  kvl::DevicePlan dp;
};

KVL_EXPORT int kvl_mla_attend_plan_create(KvlMlaAttendPlan **plan, int batch, const int *seq_len,
                                          const int64_t *seq_row0, int num_heads, int kv_lora_rank, int max_ctas) {
  if (!plan || batch <= 0 || !seq_len || !seq_row0 || num_heads <= 0 || kv_lora_rank <= 0 || max_ctas < 0) {
    set_err("invalid plan arguments");
    return -1;
  }
  *plan = nullptr;
  const int dev = current_device();
  if (dev < 0) return -1;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  HostPlan hp;
  std::vector<long long> r0(seq_row0, seq_row0 + batch);
  if (build_attend_plan(hp, batch, seq_len, r0.data(), max_ctas > 0 ? max_ctas : sms) != 0) {
    set_err("invalid sequence lengths or rows");
    return -1;
  }
  KvlMlaAttendPlan *p = new KvlMlaAttendPlan();
  p->device = dev;
  p->nh = num_heads;
  p->R = kv_lora_rank;
  if (p->dp.upload(hp, num_heads, kv_lora_rank, nullptr, nullptr, 0) != 0 || cudaDeviceSynchronize() != cudaSuccess) {
    set_err("plan upload failed");
    p->dp.release();
    delete p;
    return -1;
  }
  *plan = p;
  return 0;
}

KVL_EXPORT void kvl_mla_attend_plan_destroy(KvlMlaAttendPlan *plan) {
  if (!plan) return;
  plan->dp.release();
  delete plan;
}

KVL_EXPORT int kvl_mla_attend_plan_info(const KvlMlaAttendPlan *plan, int *ctas, int *partials, int *segments) {
  if (!plan) return -1;
  if (ctas) *ctas = plan->dp.host.grid;
  if (partials) *partials = plan->dp.host.nparts;
  if (segments) *segments = static_cast<int>(plan->dp.host.segs.size());
  return 0;
}

static int attend_common(const KvlMlaAttendPlan *plan, AttendLaunch &a, int num_heads, int R, int DR,
                         void *stream) {
  if (!plan || !a.out || !a.q || a.rows <= 0 || num_heads != plan->nh || R != plan->R || DR <= 0 || (DR & 1)) {
    set_err("invalid attend arguments");
    return -1;
  }
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) != 0) {
    set_err("the absorbed query must be 16-byte aligned");
    return -1;
  }
  a.nh = num_heads;
  a.R = R;
  a.DR = DR;
  for (int b = 0; b < plan->dp.host.batch; ++b)
    if (plan->dp.host.seq_row0[b] + plan->dp.host.seq_len[b] > a.rows) {
      set_err("sequence %d extends past the pool (%lld rows)", b, static_cast<long long>(a.rows));
      return -1;
    }
  if (plan->dp.launch(a, static_cast<cudaStream_t>(stream)) != 0) {
    set_err("attend launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  return 0;
}

KVL_EXPORT int kvl_mla_attend_bf16(const KvlMlaAttendPlan *plan, float *d_out, float *d_lse, const float *d_q,
                                   const uint16_t *d_kv, int64_t rows, int num_heads, int kv_lora_rank, int rope_dim,
                                   float softmax_scale, void *stream) {
  if (!d_kv) {
    set_err("null kv pool");
    return -1;
  }
  AttendLaunch a;
  a.q8 = false;
  a.rows = rows;
  a.q = d_q;
  a.out = d_out;
  a.lse = d_lse;
  a.kv = d_kv;
  a.softmax_scale = softmax_scale;
  return attend_common(plan, a, num_heads, kv_lora_rank, rope_dim, stream);
}

KVL_EXPORT int kvl_mla_attend_bf16_exchange(const KvlMlaAttendPlan *plan, KvlMlaPeerGroup *group, float *d_out,
                                            float *d_lse, const float *d_q, const uint16_t *d_kv, int64_t rows,
                                            float softmax_scale, void *stream) {
  if (!plan || !group || !group->connected || !d_kv || !d_out) {
    set_err("invalid attend exchange arguments");
    return -1;
  }
  if (plan->nh != kHeads || plan->R != kLatent || group->nh != plan->nh || group->R != plan->R ||
      group->batch != plan->dp.host.batch || (reinterpret_cast<uintptr_t>(d_out) & 15) != 0) {
    set_err("attend exchange: plan and group must both be %d heads x %d, the same batch, d_out 16-byte aligned",
            kHeads, kLatent);
    return -1;
  }
  AttendLaunch a;
  a.q8 = false;
  a.rows = rows;
  a.q = d_q;
  a.out = group->stage;  // unsplit sequences land here; split ones stay partials
  a.lse = group->stage + static_cast<long long>(group->batch) * group->nh * group->R;
  a.kv = d_kv;
  a.softmax_scale = softmax_scale;
  a.skip_merge = true;
  if (attend_common(plan, a, kHeads, kLatent, kRope, stream) != 0) return -1;
  if (launch_attend_exchange(group, plan->dp, d_out, d_lse, static_cast<cudaStream_t>(stream)) != cudaSuccess) {
    set_err("attend exchange launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  return 0;
}

KVL_EXPORT int kvl_mla_attend_q8(const KvlMlaAttendPlan *plan, float *d_out, float *d_lse, const float *d_q,
                                 const int8_t *d_latent_q8, const float *d_latent_scale, const uint16_t *d_rope_bf16,
                                 int64_t rows, int num_heads, int kv_lora_rank, int rope_dim, float softmax_scale,
                                 void *stream) {
  if (!d_latent_q8 || !d_latent_scale || !d_rope_bf16) {
    set_err("null q8 pool");
    return -1;
  }
  AttendLaunch a;
  a.q8 = true;
  a.rows = rows;
  a.q = d_q;
  a.out = d_out;
  a.lse = d_lse;
  a.lat8 = d_latent_q8;
  a.lscale = d_latent_scale;
  a.rope16 = d_rope_bf16;
  a.softmax_scale = softmax_scale;
  return attend_common(plan, a, num_heads, kv_lora_rank, rope_dim, stream);
}

KVL_EXPORT int kvl_mla_attend_check(const KvlMlaAttendPlan *plan, void *stream) {
  if (!plan) return -1;
  CK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  uint32_t err = 0;
  CK(cudaMemcpy(&err, plan->dp.err_word(), 4, cudaMemcpyDeviceToHost));
  if (err) {
    CK(cudaMemset(plan->dp.err_word(), 0, 4));
    set_err("attend kernel reported device error 0x%x", err);
    return -1;
  }
  return 0;
}

KVL_EXPORT int kvl_mla_merge_partials(float *d_out, float *d_lse, const float *d_part_o, const float *d_part_lse,
                                      int parts, int batch, int num_heads, int kv_lora_rank, void *stream) {
  if (!d_out || !d_part_o || !d_part_lse || parts <= 0 || batch <= 0 || num_heads <= 0 || kv_lora_rank <= 0) {
    set_err("invalid merge arguments");
    return -1;
  }
  CK(launch_merge(d_out, d_lse, d_part_o, d_part_lse, nullptr, batch, num_heads, kv_lora_rank,
                  static_cast<cudaStream_t>(stream), parts));
  return 0;
}

// =================================================================== batched decode step
// Split-K parts of the decode-step projections on the tensor-core path: a
// batch of B <= 256 tokens gives q_proj, kv_a_proj and o_proj only
// 2 x (12, 3, 8) output tiles, so the K range is split to occupy the SMs.
constexpr int kStepQSplit = 4, kStepKvaSplit = 8, kStepOSplit = 8;

// Largest split <= want that divides ksteps.
static int pick_split(int ksteps, int want) {
  for (int s = want; s > 1; --s)
    if (ksteps % s == 0) return s;
  return 1;
}

// Decode-step scratch (256-byte aligned slots): [0] q fp32 [B][NH][QD]
// (kStepQSplit partials on the tensor-core path), [1] ka fp32 [B][R+DR] (matvec path),
// [2] qabs fp32 [B][NH][R+DR], [3] mix fp32 [B][NH][R], [4] ho fp32 [B][NH*DV]
// (bf16 on the tensor-core path), [5] x bf16 [B][H], [6] q_nope bf16
// [NH][B][DN], [7] unused (0 bytes), [8] mix bf16 [NH][B][R],
// [9] kv_a partials [kStepKvaSplit][B][R+DR], [10] o_proj partials
// [kStepOSplit][B][H].
static size_t step_ws_layout(const KvlMlaConfig &c, int B, size_t off[12]) {
  const size_t NH = c.num_heads, QD = c.qk_nope_dim + c.qk_rope_dim, R = c.kv_lora_rank, DR = c.qk_rope_dim;
  const size_t DV = c.v_head_dim, DN = c.qk_nope_dim, H = c.hidden_size;
  const size_t sz[11] = {kStepQSplit * B * NH * QD * 4, B * (R + DR) * 4, B * NH * (R + DR) * 4, B * NH * R * 4,
                         B * NH * DV * 4, B * H * 2, B * NH * DN * 2, 0, B * NH * R * 2,
                         kStepKvaSplit * B * (R + DR) * 4, kStepOSplit * B * H * 4};
  size_t o = 0;
  for (int i = 0; i < 11; ++i) {
    off[i] = o;
    o += (sz[i] + 255) & ~size_t(255);
  }
  off[11] = o;
  return o;
}

KVL_EXPORT size_t kvl_mla_decode_step_workspace_bytes(const KvlMlaConfig *cfg, int batch) {
  if (!cfg || batch <= 0) return 0;
  size_t off[12];
  return step_ws_layout(*cfg, batch, off);
}

// Batches of at least this many sequences run their projections as tcgen05
// GEMMs (activations rounded to bf16); smaller ones use the per-token matvec
// kernels, which read each weight once per 8 tokens.
constexpr int kStepGemmBatch = 16;

static bool step_gemm_ok(const KvlMlaConfig &c, const KvlMlaDeviceWeights &w, const float *d_out, const void *ws,
                         int batch) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(w.q_proj) | reinterpret_cast<uintptr_t>(w.kv_a_proj) |
                      reinterpret_cast<uintptr_t>(w.kv_b_proj) | reinterpret_cast<uintptr_t>(w.o_proj) |
                      reinterpret_cast<uintptr_t>(d_out) | reinterpret_cast<uintptr_t>(ws);
  // 16-byte tensor-map bases and row strides, 16-byte vector stores
  return batch >= kStepGemmBatch && (a & 15) == 0 && c.hidden_size % 8 == 0 && c.qk_nope_dim % 8 == 0 &&
         c.qk_rope_dim % 8 == 0 && c.kv_lora_rank % 8 == 0 && c.v_head_dim % 8 == 0;
}

// The KV pool a decode step appends to and attends over: a bf16 pool
// [rows][R + DR], or a Q8 pool in the reference layout (int8 [rows][R], fp32
// scale [rows], bf16 rope [rows][DR]).
struct StepPool {
  uint16_t *kv = nullptr;
  int8_t *lat8 = nullptr;
  float *lscale = nullptr;
  uint16_t *rope16 = nullptr;
  bool q8() const { return lat8 != nullptr; }
};

// Appends each token's row (kv_a output, or `parts` split-K partials of it) to
// the pool at d_row[b], RoPE position d_pos[b]: bf16 rows, or the reference's
// row quantiser for a Q8 pool (src/mla_compressed_q8_state.c:111-127).
static cudaError_t step_append(const StepPool &pool, const KvlMlaConfig &cfg, const uint16_t *norm, const float *ka,
                               int B, const int64_t *d_row, const int *d_pos, int parts, long long part_stride,
                               cudaStream_t s) {
  const int R = cfg.kv_lora_rank, DR = cfg.qk_rope_dim;
  const long long *rows = reinterpret_cast<const long long *>(d_row);
  if (pool.q8())
    return append_q8(pool.lat8, pool.lscale, pool.rope16, 0, ka, norm, B, R, DR, 0, cfg.rms_eps, cfg.rope_theta, s,
                     rows, d_pos, parts, part_stride);
  return append_bf16(pool.kv, 0, ka, norm, B, R, DR, 0, cfg.rms_eps, cfg.rope_theta, nullptr, s, rows, d_pos, parts,
                     part_stride);
}

// The attend of a decode step over its plan (bf16 or Q8 kernel).
static int step_attend(const KvlMlaAttendPlan *plan, const StepPool &pool, const KvlMlaConfig &cfg, float *mix,
                       const float *qabs, int64_t rows, cudaStream_t s) {
  AttendLaunch a;
  a.q8 = pool.q8();
  a.rows = rows;
  a.q = qabs;
  a.out = mix;
  a.kv = pool.kv;
  a.lat8 = pool.lat8;
  a.lscale = pool.lscale;
  a.rope16 = pool.rope16;
  a.softmax_scale = 1.0f / sqrtf(static_cast<float>(cfg.qk_nope_dim + cfg.qk_rope_dim));
  a.q_dependent = true;  // qabs comes from the absorb kernel just before (absorb or gemm_absorb)
  return attend_common(plan, a, cfg.num_heads, cfg.kv_lora_rank, cfg.qk_rope_dim, s);
}

// Tensor-core projections of one decode step (batch >= kStepGemmBatch).
static int decode_step_gemm(const KvlMlaConfig &cfg, const KvlMlaDeviceWeights &w, const KvlMlaAttendPlan *plan,
                            float *d_out, const float *d_x, const StepPool &pool, int64_t rows, const int64_t *d_row,
                            const int *d_pos, int B, uint8_t *ws, const size_t *off, cudaStream_t s) {
  const uint64_t H = cfg.hidden_size, NH = cfg.num_heads, DN = cfg.qk_nope_dim, DR = cfg.qk_rope_dim;
  const uint64_t DV = cfg.v_head_dim, R = cfg.kv_lora_rank, QD = DN + DR, b = B;
  float *q = reinterpret_cast<float *>(ws + off[0]);
  float *qabs = reinterpret_cast<float *>(ws + off[2]);
  float *mix = reinterpret_cast<float *>(ws + off[3]);
  uint16_t *hob = reinterpret_cast<uint16_t *>(ws + off[4]);
  uint16_t *xb = reinterpret_cast<uint16_t *>(ws + off[5]);
  uint16_t *qn = reinterpret_cast<uint16_t *>(ws + off[6]);
  uint16_t *mixb = reinterpret_cast<uint16_t *>(ws + off[8]);
  float *ka_parts = reinterpret_cast<float *>(ws + off[9]);
  float *o_parts = reinterpret_cast<float *>(ws + off[10]);
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));

  CK(bf16_rne(xb, d_x, static_cast<long long>(b * H), s));
  GemmParams g;
  memset(&g, 0, sizeof g);
  g.err = plan->dp.err_word();  // a bounded wait that ran out: reported by kvl_mla_attend_check
  g.prefetch_b = 1;             // every B operand of the step is a weight
  // q = x Wq^T fp32 [B][NH*QD]; ka = x Wkva^T fp32 [B][R+DR]
  if (!bf16_map(&g.tm_a, xb, H, b, H * 2, 128) || !bf16_map(&g.tm_b, w.q_proj, H, NH * QD, H * 2, 256)) {
    set_err("decode step: tensor map (q_proj)");
    return -1;
  }
  const int hsteps = static_cast<int>((H + 63) / 64);
  g.M = B;
  g.N = static_cast<int>(NH * QD);
  g.K = static_cast<int>(H);
  g.c = q;
  g.ldc = g.N;
  g.ksplit = pick_split(hsteps, kStepQSplit);
  g.c_bstride = static_cast<long long>(b * NH * QD);
  const int q_parts = g.ksplit;
  CK(launch_gemm(g, 256, EPI_F32, sms, s, "gemm_q", true));
  if (!bf16_map(&g.tm_b, w.kv_a_proj, H, R + DR, H * 2, 192)) {
    set_err("decode step: tensor map (kv_a_proj)");
    return -1;
  }
  g.N = static_cast<int>(R + DR);
  g.c = ka_parts;
  g.ldc = g.N;
  g.ksplit = pick_split(hsteps, kStepKvaSplit);
  g.c_bstride = static_cast<long long>(b * (R + DR));
  CK(launch_gemm(g, 192, EPI_F32, sms, s, "gemm_kva", true));
  // the append sums the split-K partials of its row itself
  CK(step_append(pool, cfg, w.kv_a_norm, ka_parts, B, d_row, d_pos, g.ksplit, g.c_bstride, s));
  g.ksplit = 0;
  g.c_bstride = 0;
  CK(q_split(qn, qabs, q, q_parts, static_cast<long long>(b * NH * QD), B, static_cast<int>(NH),
             static_cast<int>(DN), static_cast<int>(DR), static_cast<int>(R), cfg.rope_theta, d_pos, s));
  // qabs[:, h, :R] = q_nope[:, h] . W_UK[h]   (NH products, M = B, N = R, K = DN);
  // W_UK[h] ([DN][R], rows h (DN + DV) + d of kv_b_proj) is read in place as
  // an MN-major B operand
  {
    const uint64_t ad[3] = {DN, b, NH}, as[2] = {DN * 2, b * DN * 2};
    const uint64_t bd[3] = {R, DN, NH}, bs[2] = {R * 2, (DN + DV) * R * 2};
    const uint32_t abox[3] = {64, 128, 1}, bbox[3] = {64, 64, 1};
    if (!make_tmap_3d(&g.tm_a, qn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ad, as, abox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_3d(&g.tm_b, w.kv_b_proj, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, bd, bs, bbox,
                      CU_TENSOR_MAP_SWIZZLE_128B)) {
      set_err("decode step: tensor map (absorb)");
      return -1;
    }
  }
  g.N = static_cast<int>(R);
  g.K = static_cast<int>(DN);
  g.c = qabs;
  g.ldc = static_cast<int>(NH * (R + DR));
  g.batch = static_cast<int>(NH);
  g.c_bstride = static_cast<long long>(R + DR);
  g.b_mn = 1;
  CK(launch_gemm(g, 256, EPI_F32, sms, s, "gemm_absorb", true));
  g.b_mn = 0;

  if (step_attend(plan, pool, cfg, mix, qabs, rows, s) != 0) return -1;

  // ho[:, h, :] = mix[:, h] . W_UV[h]^T   (NH products, M = B, N = DV, K = R), bf16
  CK(mix_heads_bf16(mixb, mix, B, static_cast<int>(NH), static_cast<int>(R), s));
  {
    const uint64_t ad[3] = {R, b, NH}, as[2] = {R * 2, b * R * 2};
    const uint64_t bd[3] = {R, DV, NH}, bs[2] = {R * 2, (DN + DV) * R * 2};
    const uint32_t abox[3] = {64, 128, 1}, bbox[3] = {64, 128, 1};
    if (!make_tmap_3d(&g.tm_a, mixb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ad, as, abox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_3d(&g.tm_b, w.kv_b_proj + DN * R, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, bd, bs, bbox,
                      CU_TENSOR_MAP_SWIZZLE_128B)) {
      set_err("decode step: tensor map (v up-projection)");
      return -1;
    }
  }
  g.N = static_cast<int>(DV);
  g.K = static_cast<int>(R);
  g.c = hob;
  g.ldc = static_cast<int>(NH * DV);
  g.c_bstride = static_cast<long long>(DV);
  CK(launch_gemm(g, 128, EPI_BF16, sms, s, "gemm_vup", true));

  // out = ho Wo^T fp32 [B][H]
  g.batch = 0;
  g.c_bstride = 0;
  if (!bf16_map(&g.tm_a, hob, NH * DV, b, NH * DV * 2, 128) ||
      !bf16_map(&g.tm_b, w.o_proj, NH * DV, H, NH * DV * 2, 256)) {
    set_err("decode step: tensor map (o_proj)");
    return -1;
  }
  g.N = static_cast<int>(H);
  g.K = static_cast<int>(NH * DV);
  g.c = o_parts;
  g.ldc = static_cast<int>(H);
  g.ksplit = pick_split(static_cast<int>((NH * DV + 63) / 64), kStepOSplit);
  g.c_bstride = static_cast<long long>(b * H);
  CK(launch_gemm(g, 256, EPI_F32, sms, s, "gemm_o", true));
  CK(sum_parts(d_out, o_parts, g.ksplit, g.c_bstride, static_cast<long long>(b * H), s));
  return 0;
}

// One decode step over either pool format (the arguments are checked by the
// entry points).
static int decode_step(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, const KvlMlaAttendPlan *plan,
                       float *d_out, const float *d_x, const StepPool &pool, int64_t rows, const int64_t *d_row,
                       const int *d_pos, int batch, void *d_workspace, void *stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int H = cfg->hidden_size, NH = cfg->num_heads, DN = cfg->qk_nope_dim, DR = cfg->qk_rope_dim;
  const int DV = cfg->v_head_dim, R = cfg->kv_lora_rank, QD = DN + DR;
  size_t off[12];
  step_ws_layout(*cfg, batch, off);
  uint8_t *ws = static_cast<uint8_t *>(d_workspace);
  if (step_gemm_ok(*cfg, *w, d_out, ws, batch))
    return decode_step_gemm(*cfg, *w, plan, d_out, d_x, pool, rows, d_row, d_pos, batch, ws, off, s);
  float *q = reinterpret_cast<float *>(ws + off[0]);
  float *ka = reinterpret_cast<float *>(ws + off[1]);
  float *qabs = reinterpret_cast<float *>(ws + off[2]);
  float *mix = reinterpret_cast<float *>(ws + off[3]);
  float *ho = reinterpret_cast<float *>(ws + off[4]);
  CK(gemv_bf16(q, d_x, w->q_proj, H, NH * QD, batch, s));
  CK(gemv_bf16(ka, d_x, w->kv_a_proj, H, R + DR, batch, s, true));
  CK(step_append(pool, *cfg, w->kv_a_norm, ka, batch, d_row, d_pos, 1, 0, s));
  CK(absorb(qabs, q, w->kv_b_proj, batch, NH, DN, DV, DR, R, 0, cfg->rope_theta, s, d_pos));
  if (step_attend(plan, pool, *cfg, mix, qabs, rows, s) != 0) return -1;
  CK(vup(ho, mix, w->kv_b_proj, batch, NH, DN, DV, R, s));
  CK(gemv_bf16(d_out, ho, w->o_proj, NH * DV, H, batch, s));
  return 0;
}

KVL_EXPORT int kvl_mla_decode_step_bf16(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w,
                                        const KvlMlaAttendPlan *plan, float *d_out, const float *d_x, uint16_t *d_kv,
                                        int64_t rows, const int64_t *d_row, const int *d_pos, int batch,
                                        void *d_workspace, void *stream) {
  if (!cfg || !w || !plan || !d_out || !d_x || !d_kv || !d_row || !d_pos || batch <= 0 || !d_workspace ||
      !cfg_dims_ok(*cfg) || plan->dp.host.batch != batch) {
    set_err("invalid decode step arguments");
    return -1;
  }
  StepPool pool;
  pool.kv = d_kv;
  return decode_step(cfg, w, plan, d_out, d_x, pool, rows, d_row, d_pos, batch, d_workspace, stream);
}

// Reference: src/mla_compressed_q8_state.c:161-255 (one token of one state);
// here a batch of states in one Q8 pool.
KVL_EXPORT int kvl_mla_decode_step_q8(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w,
                                      const KvlMlaAttendPlan *plan, float *d_out, const float *d_x,
                                      int8_t *d_latent_q8, float *d_latent_scale, uint16_t *d_rope_bf16,
                                      int64_t rows, const int64_t *d_row, const int *d_pos, int batch,
                                      void *d_workspace, void *stream) {
  if (!cfg || !w || !plan || !d_out || !d_x || !d_latent_q8 || !d_latent_scale || !d_rope_bf16 || !d_row ||
      !d_pos || batch <= 0 || !d_workspace || !cfg_dims_ok(*cfg) || plan->dp.host.batch != batch) {
    set_err("invalid Q8 decode step arguments");
    return -1;
  }
  StepPool pool;
  pool.lat8 = d_latent_q8;
  pool.lscale = d_latent_scale;
  pool.rope16 = d_rope_bf16;
  return decode_step(cfg, w, plan, d_out, d_x, pool, rows, d_row, d_pos, batch, d_workspace, stream);
}

KVL_EXPORT int kvl_mla_merge_packed(float *d_out, float *d_lse, const float *d_parts, int parts, int batch,
                                    int num_heads, int kv_lora_rank, void *stream) {
  if (!d_out || !d_parts || parts <= 0 || batch <= 0 || num_heads <= 0 || kv_lora_rank <= 0 ||
      (reinterpret_cast<uintptr_t>(d_parts) & 3)) {
    set_err("invalid merge arguments");
    return -1;
  }
  CK(launch_merge_packed(d_out, d_lse, d_parts, parts, batch, num_heads, kv_lora_rank,
                         static_cast<cudaStream_t>(stream)));
  return 0;
}

// =================================================================== Q8 helpers
KVL_EXPORT int kvl_mla_q8_quantize_rows(int8_t *d_q, float *d_scale, const float *d_x, int rows, int R, void *stream) {
  if (!d_q || !d_scale || !d_x || rows <= 0 || R <= 0) {
    set_err("invalid quantize arguments");
    return -1;
  }
  CK(quantize_rows(d_q, d_scale, d_x, rows, R, static_cast<cudaStream_t>(stream)));
  return 0;
}

KVL_EXPORT int kvl_mla_q8_dequant(float *d_out, const int8_t *d_q, const float *d_scale, int64_t rows, int R,
                                  void *stream) {
  if (!d_out || !d_q || !d_scale || rows <= 0 || R <= 0) {
    set_err("invalid dequant arguments");
    return -1;
  }
  CK(dequant(d_out, d_q, d_scale, rows, R, static_cast<cudaStream_t>(stream)));
  return 0;
}

KVL_EXPORT int kvl_mla_bf16_rne(uint16_t *d_out, const float *d_x, int64_t n, void *stream) {
  if (!d_out || !d_x || n <= 0) {
    set_err("invalid bf16 arguments");
    return -1;
  }
  CK(bf16_rne(d_out, d_x, n, static_cast<cudaStream_t>(stream)));
  return 0;
}
