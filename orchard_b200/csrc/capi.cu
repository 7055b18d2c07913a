// C ABI glue: status strings, device selection, buffers, and the quantised-GEMM entry
// points (surface GEMV/GEMM and the fused decode projections).
#include <sys/stat.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "qgemm.cuh"

namespace orch {

static thread_local std::string g_last_error;
static int g_sms[64] = {};
static uint32_t* g_check[64] = {};
static std::mutex g_mu;

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}
int cuda_status(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return ORCH_ERR_CUDA;
}
int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, what);
  return ORCH_OK;
}
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ORCHARD_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}
int device_index() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}
static int ensure_device_state(int d) {
  if (d < 0 || d >= 64) return fail(ORCH_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[d] == 0) {
    int v = 0;
    ORCH_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d));
    g_sms[d] = v;
  }
  if (g_check[d] == nullptr) {
    void* p = nullptr;
    ORCH_CUDA(cudaMalloc(&p, 256));
    ORCH_CUDA(cudaMemset(p, 0, 256));
    g_check[d] = static_cast<uint32_t*>(p);
    sk_preallocate(d, g_sms[d]);
  }
  return ORCH_OK;
}
int num_sms() {
  const int d = device_index();
  if (d < 0 || d >= 64) return 148;
  if (g_sms[d] == 0 && ensure_device_state(d) != ORCH_OK) return 148;
  return g_sms[d];
}
uint32_t* device_check_word() {
  const int d = device_index();
  if (d < 0 || d >= 64) return nullptr;
  if (g_check[d] == nullptr && ensure_device_state(d) != ORCH_OK) return nullptr;
  return g_check[d];
}

}  // namespace orch

using namespace orch;

extern "C" int orch_version(void) { return 100; }

extern "C" const char* orch_status_string(int status) {
  switch (status) {
    case ORCH_OK: return "ok";
    case ORCH_ERR_INVALID: return "invalid argument";
    case ORCH_ERR_CUDA: return "CUDA error";
    case ORCH_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case ORCH_ERR_NOT_INITIALIZED: return "not initialized";
    case ORCH_ERR_TIMEOUT: return "device wait timed out";
    case ORCH_ERR_DEVICE_CHECK: return "device-side input check failed";
    default: return "unknown status";
  }
}

extern "C" const char* orch_last_error(void) { return g_last_error.c_str(); }

extern "C" int orch_init(int device, const char* resource_path) {
  if (resource_path != nullptr && resource_path[0] != '\0') {
    struct stat sb;
    if (stat(resource_path, &sb) != 0 || !S_ISDIR(sb.st_mode))
      return fail(ORCH_ERR_INVALID, std::string("resource_path is not a directory: ") + resource_path);
  }
  int n = 0;
  ORCH_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(ORCH_ERR_INVALID, "device index out of range");
  ORCH_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  ORCH_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10) return fail(ORCH_ERR_UNSUPPORTED, "liborchard_b200 needs an sm_100 (Blackwell) device");
  return ensure_device_state(device);
}

extern "C" int orch_is_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  const int d = device_index();
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, d < 0 ? 0 : d) != cudaSuccess) return 0;
  return prop.major >= 10 ? 1 : 0;
}

extern "C" int orch_device_name(char* buf, size_t len) {
  ORCH_REQUIRE(buf && len > 0, "device_name: bad buffer");
  const int d = device_index();
  cudaDeviceProp prop;
  ORCH_CUDA(cudaGetDeviceProperties(&prop, d < 0 ? 0 : d));
  std::snprintf(buf, len, "%s", prop.name);
  return ORCH_OK;
}

extern "C" int orch_device_check(uint32_t* flags_out, void* stream) {
  ORCH_REQUIRE(flags_out, "device_check: null output");
  *flags_out = 0;
  const int d = device_index();
  if (d < 0 || d >= 64) return fail(ORCH_ERR_NOT_INITIALIZED, "device_check: no current device");
  cudaStream_t st = as_stream(stream);
  // The allocation-free attention entry point flags into its own word inside the library
  // (it may not allocate the shared one); report both. Reading them allocates nothing once
  // either exists.
  uint32_t* words[2] = {g_check[d], noalloc_check_word(d)};
  if (words[0] == nullptr && words[1] == nullptr) {
    words[0] = device_check_word();
    if (!words[0]) return fail(ORCH_ERR_NOT_INITIALIZED, "device_check: no device state");
  }
  for (uint32_t* w : words) {
    if (w == nullptr) continue;
    uint32_t v = 0;
    ORCH_CUDA(cudaMemcpyAsync(&v, w, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ORCH_CUDA(cudaStreamSynchronize(st));
    ORCH_CUDA(cudaMemsetAsync(w, 0, sizeof(uint32_t), st));
    ORCH_CUDA(cudaStreamSynchronize(st));
    *flags_out |= v;
  }
  return ORCH_OK;
}

extern "C" int orch_alloc(size_t bytes, void** ptr) {
  ORCH_REQUIRE(ptr, "alloc: null output");
  *ptr = nullptr;
  if (bytes == 0) bytes = 1;  // the reference creates a (tiny) buffer for empty tensors
  ORCH_CUDA(cudaMalloc(ptr, bytes));
  return ORCH_OK;
}
extern "C" int orch_free(void* ptr) {
  if (ptr) ORCH_CUDA(cudaFree(ptr));
  return ORCH_OK;
}
extern "C" int orch_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ORCH_OK;
  ORCH_REQUIRE(dst && src, "h2d: null pointer");
  ORCH_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
  return ORCH_OK;
}
extern "C" int orch_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ORCH_OK;
  ORCH_REQUIRE(dst && src, "d2h: null pointer");
  cudaStream_t st = as_stream(stream);
  ORCH_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st));
  ORCH_CUDA(cudaStreamSynchronize(st));
  return ORCH_OK;
}
extern "C" int orch_memset(void* dst, int value, size_t bytes, void* stream) {
  if (bytes == 0) return ORCH_OK;
  ORCH_REQUIRE(dst, "memset: null pointer");
  ORCH_CUDA(cudaMemsetAsync(dst, value, bytes, as_stream(stream)));
  return ORCH_OK;
}
extern "C" int orch_sync(void* stream) {
  ORCH_CUDA(cudaStreamSynchronize(as_stream(stream)));
  return ORCH_OK;
}

// ---- quantised GEMM entry points -------------------------------------------------------------
static int check_wx(const void* w, const void* s, const void* x, uint32_t K) {
  ORCH_REQUIRE(w && s && x, "quantised GEMM: null pointer");
  if (K == 0 || K % 32 != 0) return fail(ORCH_ERR_UNSUPPORTED, "quantised GEMM: K must be a positive multiple of 32");
  ORCH_REQUIRE(((uintptr_t)w & 15) == 0, "quantised GEMM: weights must be 16-byte aligned");
  ORCH_REQUIRE(((uintptr_t)x & 15) == 0, "quantised GEMM: activations must be 16-byte aligned");
  return ORCH_OK;
}

static QArgs base_args(const void* w, const void* s, const void* x, int x_dt, uint32_t M, uint32_t K,
                       uint32_t N) {
  QArgs a;
  std::memset(&a, 0, sizeof(a));
  a.w = static_cast<const uint8_t*>(w);
  a.s = static_cast<const __half*>(s);
  a.x = x;
  a.x_f32 = x_dt == ORCH_F32;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  return a;
}

extern "C" int orch_gemm_q4_0_ex(const void* w, const void* scales, const void* in, int in_dt, void* out,
                                 int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream) {
  if (B == 0 || N == 0) return ORCH_OK;
  int rc = check_wx(w, scales, in, K);
  if (rc) return rc;
  ORCH_REQUIRE(out, "gemm_q4_0: null output");
  ORCH_REQUIRE((in_dt == ORCH_F16 || in_dt == ORCH_F32) && (out_dt == ORCH_F16 || out_dt == ORCH_F32),
               "gemm_q4_0: bad dtype");
  QArgs a = base_args(w, scales, in, in_dt, B, K, N);
  a.out = out;
  a.out_f32 = out_dt == ORCH_F32;
  a.ldo = (int)N;
  return qgemm_run<W_Q4, EPI_STORE>(a, as_stream(stream));
}

extern "C" int orch_gemm_q4_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                              uint32_t N, uint32_t B, void* stream) {
  return orch_gemm_q4_0_ex(w, scales, in, ORCH_F16, out, ORCH_F16, K, N, B, stream);
}

extern "C" int orch_gemv_q4_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                              uint32_t N, void* stream) {
  return orch_gemm_q4_0_ex(w, scales, in, ORCH_F16, out, ORCH_F16, K, N, 1, stream);
}

extern "C" int orch_gemm_q8_0_ex(const void* w, const void* scales, const void* in, int in_dt, void* out,
                                 int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream) {
  if (B == 0 || N == 0) return ORCH_OK;
  int rc = check_wx(w, scales, in, K);
  if (rc) return rc;
  ORCH_REQUIRE(out, "gemm_q8_0: null output");
  QArgs a = base_args(w, scales, in, in_dt, B, K, N);
  a.out = out;
  a.out_f32 = out_dt == ORCH_F32;
  a.ldo = (int)N;
  return qgemm_run<W_Q8G, EPI_STORE>(a, as_stream(stream));
}

extern "C" int orch_gemv_q8_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                              uint32_t N, void* stream) {
  return orch_gemm_q8_0_ex(w, scales, in, ORCH_F16, out, ORCH_F16, K, N, 1, stream);
}

extern "C" int orch_gemm_q8_pc(const void* w, const void* scales, const void* in, int in_dt, void* out,
                               int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream) {
  if (B == 0 || N == 0) return ORCH_OK;
  int rc = check_wx(w, scales, in, K);
  if (rc) return rc;
  ORCH_REQUIRE(out, "gemm_q8_pc: null output");
  QArgs a = base_args(w, scales, in, in_dt, B, K, N);
  a.out = out;
  a.out_f32 = out_dt == ORCH_F32;
  a.ldo = (int)N;
  return qgemm_run<W_Q8PC, EPI_STORE>(a, as_stream(stream));
}

static int set_lora(QArgs& a, const float* t, const float* b, uint32_t r) {
  ORCH_REQUIRE(t == nullptr || (b != nullptr && r > 0), "LoRA: lora_t needs lora_b and r > 0");
  a.lora_t = t;
  a.lora_b = b;
  a.lora_r = (int)r;
  return ORCH_OK;
}

// Weights of the fused entry points: reference layout (w + scales) or tiled (scales null).
static int check_q4w(const void* w, const void* s, const void* x, uint32_t K, bool tiled) {
  if (!tiled) return check_wx(w, s, x, K);
  ORCH_REQUIRE(w && x, "tiled INT4 GEMM: null pointer");
  if (K == 0 || K % 32 != 0) return fail(ORCH_ERR_UNSUPPORTED, "tiled INT4 GEMM: K must be a positive multiple of 32");
  ORCH_REQUIRE(((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0, "tiled INT4 GEMM: buffers must be 16-byte aligned");
  return ORCH_OK;
}

static int linear_resid(const void* w, const void* scales, bool tiled, const void* x, float* resid, uint32_t M,
                        uint32_t K, uint32_t N, const float* lora_t, const float* lora_b, uint32_t lora_r,
                        void* stream) {
  if (M == 0 || N == 0) return ORCH_OK;
  int rc = check_q4w(w, scales, x, K, tiled);
  if (rc) return rc;
  ORCH_REQUIRE(resid, "q4_linear_resid: null residual");
  QArgs a = base_args(w, scales, x, ORCH_F16, M, K, N);
  a.tiled = tiled;
  a.out = resid;
  a.out_f32 = 1;
  a.ldo = (int)N;
  if ((rc = set_lora(a, lora_t, lora_b, lora_r))) return rc;
  return qgemm_run<W_Q4, EPI_RESID>(a, as_stream(stream));
}

static int linear_swiglu(const void* w13, const void* s13, bool tiled, const void* x, void* h, uint32_t M, uint32_t K,
                         uint32_t F, const float* lora_t, const float* lora_b, uint32_t lora_r, void* stream) {
  if (M == 0 || F == 0) return ORCH_OK;
  int rc = check_q4w(w13, s13, x, K, tiled);
  if (rc) return rc;
  ORCH_REQUIRE(h, "q4_linear_swiglu: null output");
  if (F % 16 != 0) return fail(ORCH_ERR_UNSUPPORTED, "q4_linear_swiglu: F must be a multiple of 16");
  QArgs a = base_args(w13, s13, x, ORCH_F16, M, K, 2 * F);
  a.tiled = tiled;
  a.out = h;
  if ((rc = set_lora(a, lora_t, lora_b, lora_r))) return rc;
  return qgemm_run<W_Q4, EPI_SWIGLU>(a, as_stream(stream));
}

static int qkv_rope(const void* wqkv, const void* sqkv, bool tiled, const void* x, uint32_t M, uint32_t K, uint32_t H,
                    uint32_t num_heads, const int32_t* pos, const int32_t* slots, const float* cos_tab,
                    const float* sin_tab, uint32_t max_pos, void* q_out, void* k_cache, void* v_cache,
                    uint32_t max_seq, uint32_t num_slots, const float* lora_t, const float* lora_b, uint32_t lora_r,
                    void* stream) {
  if (M == 0) return ORCH_OK;
  int rc = check_q4w(wqkv, sqkv, x, K, tiled);
  if (rc) return rc;
  ORCH_REQUIRE(pos && cos_tab && sin_tab && q_out && k_cache && v_cache, "q4_qkv_rope: null pointer");
  ORCH_REQUIRE(num_heads > 0 && H % num_heads == 0, "q4_qkv_rope: H must be a multiple of num_heads");
  const uint32_t hd = H / num_heads;
  ORCH_REQUIRE(hd % 2 == 0, "q4_qkv_rope: head_dim must be even");
  ORCH_REQUIRE(H < 65536, "q4_qkv_rope: H must be below 65536");
  ORCH_REQUIRE(max_seq > 0 && max_pos > 0 && num_slots > 0, "q4_qkv_rope: empty cache");
  ORCH_REQUIRE(num_slots <= 0x7fffffffu, "q4_qkv_rope: num_slots out of range");
  QArgs a = base_args(wqkv, sqkv, x, ORCH_F16, M, K, 3 * H);
  a.tiled = tiled;
  a.out = q_out;
  a.H = (int)H;
  a.nh = (int)num_heads;
  a.hd = (int)hd;
  a.hd_magic = (uint32_t)((0x100000000ull + hd - 1) / hd);
  a.max_seq = (int)max_seq;
  a.num_slots = (int)num_slots;
  a.max_pos = (int)max_pos;
  a.pos = pos;
  a.slots = slots;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.kc = static_cast<__half*>(k_cache);
  a.vc = static_cast<__half*>(v_cache);
  if ((rc = set_lora(a, lora_t, lora_b, lora_r))) return rc;
  return qgemm_run<W_Q4, EPI_QKV>(a, as_stream(stream));
}

extern "C" int orch_q4_linear_resid(const void* w, const void* scales, const void* x, float* resid,
                                    uint32_t M, uint32_t K, uint32_t N, const float* lora_t,
                                    const float* lora_b, uint32_t lora_r, void* stream) {
  return linear_resid(w, scales, false, x, resid, M, K, N, lora_t, lora_b, lora_r, stream);
}

extern "C" int orch_q4_linear_swiglu(const void* w13, const void* s13, const void* x, void* h, uint32_t M,
                                     uint32_t K, uint32_t F, const float* lora_t, const float* lora_b,
                                     uint32_t lora_r, void* stream) {
  return linear_swiglu(w13, s13, false, x, h, M, K, F, lora_t, lora_b, lora_r, stream);
}

extern "C" int orch_q4_qkv_rope(const void* wqkv, const void* sqkv, const void* x, uint32_t M, uint32_t K,
                                uint32_t H, uint32_t num_heads, const int32_t* pos, const int32_t* slots,
                                const float* cos_tab, const float* sin_tab, uint32_t max_pos, void* q_out,
                                void* k_cache, void* v_cache, uint32_t max_seq, uint32_t num_slots,
                                const float* lora_t, const float* lora_b, uint32_t lora_r, void* stream) {
  return qkv_rope(wqkv, sqkv, false, x, M, K, H, num_heads, pos, slots, cos_tab, sin_tab, max_pos, q_out, k_cache,
                  v_cache, max_seq, num_slots, lora_t, lora_b, lora_r, stream);
}

// ---- tiled-layout forms (weights re-laid by orch_q4t_pack) ----------------------------------
extern "C" int orch_q4t_gemm(const void* tiled, const void* in, void* out, int out_dt, uint32_t K, uint32_t N,
                             uint32_t M, void* stream) {
  if (M == 0 || N == 0) return ORCH_OK;
  int rc = check_q4w(tiled, nullptr, in, K, true);
  if (rc) return rc;
  ORCH_REQUIRE(out, "q4t_gemm: null output");
  ORCH_REQUIRE(out_dt == ORCH_F16 || out_dt == ORCH_F32, "q4t_gemm: bad dtype");
  QArgs a = base_args(tiled, nullptr, in, ORCH_F16, M, K, N);
  a.tiled = 1;
  a.out = out;
  a.out_f32 = out_dt == ORCH_F32;
  a.ldo = (int)N;
  return qgemm_run<W_Q4, EPI_STORE>(a, as_stream(stream));
}

extern "C" int orch_q4t_linear_resid(const void* tiled, const void* x, float* resid, uint32_t M, uint32_t K,
                                     uint32_t N, const float* lora_t, const float* lora_b, uint32_t lora_r,
                                     void* stream) {
  return linear_resid(tiled, nullptr, true, x, resid, M, K, N, lora_t, lora_b, lora_r, stream);
}

extern "C" int orch_q4t_linear_swiglu(const void* tiled13, const void* x, void* h, uint32_t M, uint32_t K,
                                      uint32_t F, const float* lora_t, const float* lora_b, uint32_t lora_r,
                                      void* stream) {
  return linear_swiglu(tiled13, nullptr, true, x, h, M, K, F, lora_t, lora_b, lora_r, stream);
}

extern "C" int orch_q4t_qkv_rope(const void* tiled_qkv, const void* x, uint32_t M, uint32_t K, uint32_t H,
                                 uint32_t num_heads, const int32_t* pos, const int32_t* slots, const float* cos_tab,
                                 const float* sin_tab, uint32_t max_pos, void* q_out, void* k_cache, void* v_cache,
                                 uint32_t max_seq, uint32_t num_slots, const float* lora_t, const float* lora_b,
                                 uint32_t lora_r, void* stream) {
  return qkv_rope(tiled_qkv, nullptr, true, x, M, K, H, num_heads, pos, slots, cos_tab, sin_tab, max_pos, q_out,
                  k_cache, v_cache, max_seq, num_slots, lora_t, lora_b, lora_r, stream);
}

// ---- RMSNorm fused in front of the tiled Q/K/V and gate/up projections ----------------------
// M <= 8 rows: the GEMV normalises the fp32 residual itself (no separate launch, xn untouched);
// more rows: RMSNorm into xn, then the tensor-core GEMM (two launches, as before).
static int rms_args(QArgs& a, const float* x, const float* norm_w, float eps) {
  ORCH_REQUIRE(x && norm_w, "rmsnorm-fused GEMM: null pointer");
  ORCH_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)norm_w & 15) == 0,
               "rmsnorm-fused GEMM: x and norm_w must be 16-byte aligned");
  a.x = x;
  a.x_f32 = 1;
  a.norm_w = norm_w;
  a.norm_eps = eps;
  return ORCH_OK;
}

extern "C" int orch_q4t_rms_qkv_rope(const void* tiled_qkv, const float* x, const float* norm_w, float eps, void* xn,
                                     uint32_t M, uint32_t K, uint32_t H, uint32_t num_heads, const int32_t* pos,
                                     const int32_t* slots, const float* cos_tab, const float* sin_tab,
                                     uint32_t max_pos, void* q_out, void* k_cache, void* v_cache, uint32_t max_seq,
                                     uint32_t num_slots, void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(xn, "rms_qkv_rope: null xn");
  if (M <= gemv_tiled_limit()) {
    // the argument checks of the unfused form, on the fp16 scratch as a stand-in for x
    int rc = check_q4w(tiled_qkv, nullptr, xn, K, true);
    if (rc) return rc;
    ORCH_REQUIRE(pos && cos_tab && sin_tab && q_out && k_cache && v_cache, "rms_qkv_rope: null pointer");
    ORCH_REQUIRE(num_heads > 0 && H % num_heads == 0 && (H / num_heads) % 2 == 0 && H < 65536,
                 "rms_qkv_rope: bad head shape");
    ORCH_REQUIRE(max_seq > 0 && max_pos > 0 && num_slots > 0 && num_slots <= 0x7fffffffu, "rms_qkv_rope: empty cache");
    QArgs a = base_args(tiled_qkv, nullptr, x, ORCH_F32, M, K, 3 * H);
    a.tiled = 1;
    if ((rc = rms_args(a, x, norm_w, eps))) return rc;
    const uint32_t hd = H / num_heads;
    a.out = q_out;
    a.H = (int)H;
    a.nh = (int)num_heads;
    a.hd = (int)hd;
    a.hd_magic = (uint32_t)((0x100000000ull + hd - 1) / hd);
    a.max_seq = (int)max_seq;
    a.num_slots = (int)num_slots;
    a.max_pos = (int)max_pos;
    a.pos = pos;
    a.slots = slots;
    a.cos_tab = cos_tab;
    a.sin_tab = sin_tab;
    a.kc = static_cast<__half*>(k_cache);
    a.vc = static_cast<__half*>(v_cache);
    rc = gemv_tiled_run<EPI_QKV>(a, as_stream(stream));
    if (rc != ORCH_ERR_UNSUPPORTED) return rc;
  }
  int rc = orch_rmsnorm_ex(x, ORCH_F32, norm_w, ORCH_F32, xn, ORCH_F16, eps, K, M, stream);
  if (rc) return rc;
  return orch_q4t_qkv_rope(tiled_qkv, xn, M, K, H, num_heads, pos, slots, cos_tab, sin_tab, max_pos, q_out, k_cache,
                           v_cache, max_seq, num_slots, nullptr, nullptr, 0, stream);
}

extern "C" int orch_q4t_rms_linear_swiglu(const void* tiled13, const float* x, const float* norm_w, float eps,
                                          void* xn, void* h, uint32_t M, uint32_t K, uint32_t F, void* stream) {
  if (M == 0 || F == 0) return ORCH_OK;
  ORCH_REQUIRE(xn && h, "rms_linear_swiglu: null pointer");
  if (F % 16 != 0) return fail(ORCH_ERR_UNSUPPORTED, "rms_linear_swiglu: F must be a multiple of 16");
  if (M <= gemv_tiled_limit()) {
    int rc = check_q4w(tiled13, nullptr, xn, K, true);
    if (rc) return rc;
    QArgs a = base_args(tiled13, nullptr, x, ORCH_F32, M, K, 2 * F);
    a.tiled = 1;
    if ((rc = rms_args(a, x, norm_w, eps))) return rc;
    a.out = h;
    rc = gemv_tiled_run<EPI_SWIGLU>(a, as_stream(stream));
    if (rc != ORCH_ERR_UNSUPPORTED) return rc;
  }
  int rc = orch_rmsnorm_ex(x, ORCH_F32, norm_w, ORCH_F32, xn, ORCH_F16, eps, K, M, stream);
  if (rc) return rc;
  return orch_q4t_linear_swiglu(tiled13, xn, h, M, K, F, nullptr, nullptr, 0, stream);
}

extern "C" uint32_t orch_gemv_max_rows(void) { return gemv_tiled_limit(); }
