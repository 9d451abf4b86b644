// Host-side helpers shared by the kernel launchers: error recording, device
// properties, the device status word and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/tfb200.h"

namespace tfb {

// The two 16-bit operand types of the tensor-core kernels: kDtF16 (IEEE
// binary16: the compute type of the fp32 model and the fp16 model's own type)
// and kDtBF16 (bfloat16 models).
constexpr int kDtF16 = 0;
constexpr int kDtBF16 = 1;

// Records a formatted message for tf_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
int last_error_code();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Streaming-multiprocessor count of the current device (cached).
int device_sm_count();

// Device address of the library's status word on the current device
// (resolved once per device); nullptr after recording an error.
int* device_status_ptr();

// 2-D fp16 tensor map, 128-byte swizzle: inner extent `inner` elements with
// row pitch `ld` elements, `outer` rows, box of box_inner x box_outer.
int make_tmap_2d_f16(CUtensorMap* map, const void* base, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer);

// 3-D fp16 tensor map (inner, rows, batches) with row pitch `ld` and batch
// pitch `bstride` (elements), 128-byte swizzle, box box_inner x box_rows x 1.
int make_tmap_3d_f16(CUtensorMap* map, const void* base, long long inner, long long rows, long long batches,
                     long long ld, long long bstride, int box_inner, int box_rows);

// Programmatic dependent launch. Every kernel of this library is launched
// with programmatic stream serialization: it may start (barrier set-up,
// TMEM allocation, tensor-map prefetch) while the previous kernel on the
// stream drains, and waits (griddepcontrol.wait) before it touches global
// memory the previous kernel may write or read. TFB_PDL=0 in the environment
// turns it off (plain stream order).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// kernels (defined in their own translation units)
struct GemmCall {
  const void* A;
  long long lda;
  const void* W;
  long long ldw;
  const float* bias;
  void* C;  // 16-bit output (epilogues 0, 1, 5)
  long long ldc;
  const void* x_in;  // residual: fp32 (epilogue 2) or the operand type (epilogue 4)
  void* x_out;
  long long ldx;
  const uint8_t* valid;
  int mask_mode;
  long long M, N, K;
  // 0 C = T(acc + bias); 1 C = T(gelu(acc + bias)); 2 fp32 residual add;
  // 4 residual add in T; 5 C = T(gelu(T(acc + bias))). T = the operand type
  int epilogue;
  int dtype;  // operand type: kDtF16 (0) or kDtBF16 (1)
  int a_repeat;
  int tile_n;
  int pair;  // 0 automatic, 1 one-CTA tiles, 2 two-SM (CTA pair) tiles
  int* ready;  // residual epilogues: per-8-row-group counts of stored columns, or null
};

// LayerNorm applied to the result of a residual projection (split-K form):
// normed = mask_out(LayerNorm(x_out) * w + b), contiguous [M, N]
struct LnFuse {
  const float* w;
  const float* b;
  float eps;
  void* normed;
  int flags;  // TF_LN_MASK_OUT, TF_LN_OUT_F32
};

int gemm_f16(const GemmCall& g, cudaStream_t stream);
// split-K GEMM (epilogues 0, 1, 2, 4, 5) with an fp32 partial-sum workspace;
// with `ln` (residual epilogues) the reduce kernel also runs that LayerNorm
int gemm_splitk_f16(const GemmCall& g, int splits, float* ws, long long ws_bytes, cudaStream_t stream,
                    const LnFuse* ln = nullptr);
long long gemm_splitk_workspace_bytes(long long M, long long N, long long K, int splits);
// the same with the library's fixed 4 MiB device scratch (no allocation)
int gemm_splitk_static_f16(const GemmCall& g, int splits, cudaStream_t stream);

int ln_residual(const void* x, const void* delta, const float* w, const float* b, float eps,
                const uint8_t* valid, long long M, int D, int flags, void* x_out, void* normed,
                cudaStream_t stream);
// LayerNorm of rows a concurrent residual GEMM is still storing (ready mode)
int ln_ready(const void* x, const float* w, const float* b, float eps, const uint8_t* valid, long long M, int D,
             int flags, void* normed, int* ready, cudaStream_t stream);

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  long long ld_q, ld_kv, bs_q, bs_kv;
  void* out;
  long long ld_o, bs_o;
  float* lse;
  const uint8_t* key_valid;
  long long batch, heads, seq_q, seq_k, head_dim;
  float scale;
  long long q_pos0, k_pos0;
  int flags;
};

int flash_fwd(const AttnArgs& a, cudaStream_t stream);

struct MergeArgs {
  float* o_acc;
  float* lse_acc;
  const float* o_part;
  const float* lse_part;
  long long ld, bs;
  void* out16;
  long long ld16, bs16;
  long long batch, heads, seq_q, head_dim;
};

int attn_merge(const MergeArgs& a, cudaStream_t stream);

// test probe of the bounded waits (probe.cu)
int wait_timeout_probe(const void* src, long long limit_ns, int* out, cudaStream_t stream);

}  // namespace tfb
