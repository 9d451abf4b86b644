// The C ABI (include/tfb200.h) and the host helpers shared by the launchers:
// error messages, per-device properties, the device status word and TMA
// tensor-map encoding through the driver entry point (no libcuda link).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include <cstdlib>

#include "launch.h"

namespace tfb {

// Status word written by kernels whose bounded waits ran out. One per device
// (every device that loads this library holds its own copy).
__device__ int g_tfb_status = 0;

namespace {
thread_local char g_msg[512] = "";
thread_local int g_code = TF_OK;

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int* status = nullptr;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

// Resolves per-device properties on first use: the device must be sm_100
// (the library holds sm_100a code only) and the status word's device address
// is looked up with the device current.
DeviceInfo* device_info() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error(TF_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error(TF_ERR_DEVICE, "device index %d out of range", dev);
    return nullptr;
  }
  DeviceInfo& di = g_dev[dev];
  if (di.ready) return &di;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (di.ready) return &di;
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) {
    set_error(TF_ERR_DEVICE, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
    return nullptr;
  }
  if (prop.major != 10 || prop.minor != 0) {
    set_error(TF_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
              prop.major, prop.minor);
    return nullptr;
  }
  void* addr = nullptr;
  e = cudaGetSymbolAddress(&addr, g_tfb_status);
  if (e != cudaSuccess) {
    set_error(TF_ERR_DEVICE, "cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
    return nullptr;
  }
  di.sms = prop.multiProcessorCount;
  di.status = static_cast<int*>(addr);
  di.ready = true;
  return &di;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  g_code = code;
  return code;
}

int last_error_code() { return g_code == TF_OK ? TF_ERR_DEVICE : g_code; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("TFB_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

int device_sm_count() {
  DeviceInfo* di = device_info();
  return di ? di->sms : 148;
}

int* device_status_ptr() {
  DeviceInfo* di = device_info();
  return di ? di->status : nullptr;
}

static int encode(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                  const cuuint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(TF_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TF_ERR_DRIVER, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return TF_OK;
}

int make_tmap_2d_f16(CUtensorMap* map, const void* base, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer) {
  if (!aligned16(base) || (ld * 2) % 16 != 0) return set_error(TF_ERR_ALIGN, "tensor map: base/pitch alignment");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  return encode(map, 2, base, dims, strides, box);
}

int make_tmap_3d_f16(CUtensorMap* map, const void* base, long long inner, long long rows, long long batches,
                     long long ld, long long bstride, int box_inner, int box_rows) {
  if (!aligned16(base) || (ld * 2) % 16 != 0 || (bstride * 2) % 16 != 0)
    return set_error(TF_ERR_ALIGN, "tensor map: base/pitch alignment");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batches)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(bstride * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
  return encode(map, 3, base, dims, strides, box);
}

}  // namespace tfb

// ---------------------------------------------------------------------------
// extern "C" entry points
// ---------------------------------------------------------------------------

using tfb::set_error;

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

static inline int begin_call() {
  tfb::g_msg[0] = '\0';
  tfb::g_code = TF_OK;
  return tfb::device_status_ptr() == nullptr ? tfb::last_error_code() : TF_OK;
}

extern "C" {

int tf_abi_version(void) { return 11; }

const char* tf_last_error(void) { return tfb::g_msg; }

int tf_device_status(int* code, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  if (code == nullptr) return set_error(TF_ERR_SHAPE, "tf_device_status: code is NULL");
  cudaError_t e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return set_error(TF_ERR_DEVICE, "stream synchronize: %s", cudaGetErrorString(e));
  int host = 0;
  e = cudaMemcpyFromSymbol(&host, tfb::g_tfb_status, sizeof(int));
  if (e != cudaSuccess) return set_error(TF_ERR_DEVICE, "read status: %s", cudaGetErrorString(e));
  const int zero = 0;
  e = cudaMemcpyToSymbol(tfb::g_tfb_status, &zero, sizeof(int));
  if (e != cudaSuccess) return set_error(TF_ERR_DEVICE, "clear status: %s", cudaGetErrorString(e));
  *code = host;
  return host == 0 ? TF_OK : set_error(TF_ERR_TIMEOUT, "a kernel wait ran out (device code %d)", host);
}

int tf_test_wait_timeout(const void* src, int64_t limit_ns, int* out, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  return tfb::wait_timeout_probe(src, limit_ns, out, as_stream(stream));
}

int tf_ln_residual(const void* x, const void* delta, const float* w, const float* b, float eps,
                   const uint8_t* valid, int64_t M, int64_t D, int flags, void* x_out, void* normed,
                   void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  if (D > (1 << 20)) return set_error(TF_ERR_SHAPE, "ln_residual: D too large");
  return tfb::ln_residual(x, delta, w, b, eps, valid, M, static_cast<int>(D), flags, x_out, normed,
                          as_stream(stream));
}

// Internal epilogue code and operand type of a tf_gemm* epilogue argument
// (TF_EPI_BIAS, TF_EPI_BIAS_GELU or TF_EPI_BIAS_GELU_ROUNDED, optionally
// with TF_EPI_BF16); -1 if it names none of them.
static int gemm_epilogue(int epilogue, int& dtype) {
  dtype = (epilogue & TF_EPI_BF16) ? tfb::kDtBF16 : tfb::kDtF16;
  switch (epilogue & 0xF) {
    case TF_EPI_BIAS: return 0;
    case TF_EPI_BIAS_GELU: return 1;
    case TF_EPI_BIAS_GELU_ROUNDED: return 5;
    default: return -1;
  }
}

// Internal residual epilogue, mask mode and operand type of a
// tf_gemm_residual* mask_mode argument; false if it is malformed.
static bool residual_mode(int mask_mode, int& epi, int& mask, int& dtype) {
  if (mask_mode & ~(3 | TF_RES_X16 | TF_RES_BF16)) return false;
  mask = mask_mode & 3;
  if (mask > 2) return false;
  epi = (mask_mode & TF_RES_X16) ? 4 : 2;
  dtype = (mask_mode & TF_RES_BF16) ? tfb::kDtBF16 : tfb::kDtF16;
  return true;
}

static int gemm_common(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C,
                       int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int tile_n, int pair,
                       void* stream) {
  if (epilogue & ~(0xF | TF_EPI_W_SPLIT | TF_EPI_BF16)) return set_error(TF_ERR_SHAPE, "tf_gemm: unknown epilogue bits");
  int dtype = 0;
  const int epi = gemm_epilogue(epilogue, dtype);
  if (epi < 0) return set_error(TF_ERR_SHAPE, "tf_gemm: epilogue %d", epilogue & 0xF);
  if ((epilogue & TF_EPI_W_SPLIT) && dtype != tfb::kDtF16)
    return set_error(TF_ERR_SHAPE, "tf_gemm: split weights are fp16 only");
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.C = C;
  g.ldc = ldc;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = (epilogue & TF_EPI_W_SPLIT) ? 2 : 1;
  g.tile_n = tile_n;
  g.pair = pair;
  return tfb::gemm_f16(g, as_stream(stream));
}

int tf_gemm(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C, int64_t ldc,
            int64_t M, int64_t N, int64_t K, int epilogue, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  return gemm_common(A, lda, W, ldw, bias, C, ldc, M, N, K, epilogue, 0, 0, stream);
}

int tf_gemm_tiled(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C,
                  int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int tile_n, int pair, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  if (tile_n != 0 && tile_n != 64 && tile_n != 128 && tile_n != 256)
    return set_error(TF_ERR_SHAPE, "tf_gemm_tiled: tile_n=%d (0, 64, 128 or 256)", tile_n);
  if (tile_n != 0 && N % tile_n != 0) return set_error(TF_ERR_SHAPE, "tf_gemm_tiled: N %% tile_n != 0");
  if (pair < 0 || pair > 2) return set_error(TF_ERR_SHAPE, "tf_gemm_tiled: pair=%d (0, 1 or 2)", pair);
  if (pair == 2 && tile_n == 64) return set_error(TF_ERR_SHAPE, "tf_gemm_tiled: 2-SM tiles are 128 or 256 wide");
  return gemm_common(A, lda, W, ldw, bias, C, ldc, M, N, K, epilogue, tile_n, pair, stream);
}

static int gemm_residual_common(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                                const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                                int64_t M, int64_t N, int64_t K, int w_split, int tile_n, int pair, int* ready,
                                void* stream) {
  int epi = 0, mask = 0, dtype = 0;
  if (!residual_mode(mask_mode, epi, mask, dtype))
    return set_error(TF_ERR_SHAPE, "tf_gemm_residual: mask_mode=%d", mask_mode);
  if (w_split && dtype != tfb::kDtF16) return set_error(TF_ERR_SHAPE, "tf_gemm_residual: split weights are fp16 only");
  if (tile_n != 0 && tile_n != 64 && tile_n != 128 && tile_n != 256)
    return set_error(TF_ERR_SHAPE, "tf_gemm_residual: tile_n=%d (0, 64, 128 or 256)", tile_n);
  if (pair < 0 || pair > 2 || (pair == 2 && tile_n == 64))
    return set_error(TF_ERR_SHAPE, "tf_gemm_residual: pair=%d with tile_n=%d", pair, tile_n);
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.x_in = x_in;
  g.x_out = x_out;
  g.ldx = ldx;
  g.valid = valid;
  g.mask_mode = mask;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = w_split ? 2 : 1;
  g.tile_n = tile_n;
  g.pair = pair;
  g.ready = ready;
  return tfb::gemm_f16(g, as_stream(stream));
}

int tf_gemm_residual(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                     const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                     int64_t M, int64_t N, int64_t K, int w_split, int tile_n, int pair, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  return gemm_residual_common(A, lda, W, ldw, bias, x_in, x_out, ldx, valid, mask_mode, M, N, K, w_split, tile_n,
                              pair, nullptr, stream);
}

int tf_gemm_residual_ready(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                           const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                           int64_t M, int64_t N, int64_t K, int w_split, int* ready, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  if (ready == nullptr || reinterpret_cast<uintptr_t>(ready) % 4 != 0)
    return set_error(TF_ERR_ALIGN, "tf_gemm_residual_ready: ready must be a non-null int32 array");
  if (ldx != N) return set_error(TF_ERR_SHAPE, "tf_gemm_residual_ready: x_out must be contiguous (ldx == N)");
  return gemm_residual_common(A, lda, W, ldw, bias, x_in, x_out, ldx, valid, mask_mode, M, N, K, w_split, 0, 0,
                              ready, stream);
}

int tf_ln_ready(const void* x, const float* w, const float* b, float eps, const uint8_t* valid, int64_t M,
                int64_t D, int flags, void* normed, int* ready, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  if (D > (1 << 20)) return set_error(TF_ERR_SHAPE, "ln_ready: D too large");
  return tfb::ln_ready(x, w, b, eps, valid, M, static_cast<int>(D), flags, normed, ready, as_stream(stream));
}

int64_t tf_gemm_splitk_workspace(int64_t M, int64_t N, int64_t K, int splits) {
  if (begin_call()) return -1;
  return tfb::gemm_splitk_workspace_bytes(M, N, K, splits);
}

int tf_gemm_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C, int64_t ldc,
                   int64_t M, int64_t N, int64_t K, int epilogue, int splits, void* workspace,
                   int64_t workspace_bytes, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  int dtype = 0;
  const int epi = (epilogue & ~(0xF | TF_EPI_BF16)) ? -1 : gemm_epilogue(epilogue, dtype);
  if (epi < 0) return set_error(TF_ERR_SHAPE, "tf_gemm_splitk: epilogue=%d", epilogue);
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.C = C;
  g.ldc = ldc;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = 1;
  return tfb::gemm_splitk_f16(g, splits, static_cast<float*>(workspace), workspace_bytes, as_stream(stream));
}

int tf_gemm_splitk_static(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C,
                          int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int splits, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  int dtype = 0;
  const int epi = (epilogue & ~(0xF | TF_EPI_BF16)) ? -1 : gemm_epilogue(epilogue, dtype);
  if (epi < 0) return set_error(TF_ERR_SHAPE, "tf_gemm_splitk_static: epilogue=%d", epilogue);
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.C = C;
  g.ldc = ldc;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = 1;
  return tfb::gemm_splitk_static_f16(g, splits, as_stream(stream));
}

int tf_gemm_residual_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                            const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                            int64_t M, int64_t N, int64_t K, int splits, void* workspace, int64_t workspace_bytes,
                            void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  int epi = 0, mask = 0, dtype = 0;
  if (!residual_mode(mask_mode, epi, mask, dtype))
    return set_error(TF_ERR_SHAPE, "tf_gemm_residual_splitk: mask_mode=%d", mask_mode);
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.x_in = x_in;
  g.x_out = x_out;
  g.ldx = ldx;
  g.valid = valid;
  g.mask_mode = mask;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = 1;
  return tfb::gemm_splitk_f16(g, splits, static_cast<float*>(workspace), workspace_bytes, as_stream(stream));
}

int tf_gemm_residual_ln_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                               const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                               int64_t M, int64_t N, int64_t K, int splits, void* workspace,
                               int64_t workspace_bytes, const float* ln_w, const float* ln_b, float eps,
                               void* normed, int ln_flags, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  int epi = 0, mask = 0, dtype = 0;
  if (!residual_mode(mask_mode, epi, mask, dtype))
    return set_error(TF_ERR_SHAPE, "tf_gemm_residual_ln_splitk: mask_mode=%d", mask_mode);
  tfb::GemmCall g = {};
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.bias = bias;
  g.x_in = x_in;
  g.x_out = x_out;
  g.ldx = ldx;
  g.valid = valid;
  g.mask_mode = mask;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epilogue = epi;
  g.dtype = dtype;
  g.a_repeat = 1;
  tfb::LnFuse ln = {ln_w, ln_b, eps, normed, ln_flags};
  return tfb::gemm_splitk_f16(g, splits, static_cast<float*>(workspace), workspace_bytes, as_stream(stream), &ln);
}

int tf_flash_fwd(const void* q, const void* k, const void* v, int64_t ld_q, int64_t ld_kv, int64_t bs_q,
                 int64_t bs_kv, void* out, int64_t ld_o, int64_t bs_o, float* lse, const uint8_t* key_valid,
                 int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k, int64_t head_dim, float scale,
                 int64_t q_pos0, int64_t k_pos0, int flags, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  tfb::AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ld_q = ld_q;
  a.ld_kv = ld_kv;
  a.bs_q = bs_q;
  a.bs_kv = bs_kv;
  a.out = out;
  a.ld_o = ld_o;
  a.bs_o = bs_o;
  a.lse = lse;
  a.key_valid = key_valid;
  a.batch = batch;
  a.heads = heads;
  a.seq_q = seq_q;
  a.seq_k = seq_k;
  a.head_dim = head_dim;
  a.scale = scale;
  a.q_pos0 = q_pos0;
  a.k_pos0 = k_pos0;
  a.flags = flags;
  return tfb::flash_fwd(a, as_stream(stream));
}

int tf_attn_merge(float* o_acc, float* lse_acc, const float* o_part, const float* lse_part, int64_t ld,
                  int64_t bs, void* out16, int64_t ld16, int64_t bs16, int64_t batch, int64_t heads,
                  int64_t seq_q, int64_t head_dim, void* stream) {
  int rc = begin_call();
  if (rc) return rc;
  tfb::MergeArgs a;
  a.o_acc = o_acc;
  a.lse_acc = lse_acc;
  a.o_part = o_part;
  a.lse_part = lse_part;
  a.ld = ld;
  a.bs = bs;
  a.out16 = out16;
  a.ld16 = ld16;
  a.bs16 = bs16;
  a.batch = batch;
  a.heads = heads;
  a.seq_q = seq_q;
  a.head_dim = head_dim;
  return tfb::attn_merge(a, as_stream(stream));
}

}  // extern "C"
