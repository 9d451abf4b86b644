// Residual add + LayerNorm, one pass over HBM.
//
//   x_new  = mask_x(x + mask_delta(fp32(delta)))     (stored when WRITE_X)
//   normed = mask_out(LayerNorm(x_new) * w + b)      (fp16, or fp32)
//
// Same operation order as the reference's _add_ln_kernel
// (torch_transformer_benchmark.py:884-962) and its ATen branch (3988-4001).
// The fp16 delta is upcast losslessly and added in fp32; mean and variance are
// the two-pass moments over the row held in registers, as the reference
// kernel does (mean first, then the centred sum of squares).
//
// Layout: one warp per row (grid-stride over rows), 8 warps per 256-thread
// block, as many blocks as are resident on the device. Each lane owns
// 8-element chunks (two float4 of x, one 16-byte vector of fp16 delta) at
// chunk index lane + 32*i, so every warp-wide load is a contiguous,
// fully-coalesced 512 B (fp32) or 256 B (fp16) segment. HBM-bound: bytes per
// row = D*(4 read x + 2 read delta + 4 write x + 2 write normed).
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kLnRowsPerBlock = 8;

template <int NCH>  // 8-element chunks per lane (row width up to 256*NCH)
__global__ void __launch_bounds__(256) ln_residual_kernel(const float* __restrict__ x,
                                                          const __half* __restrict__ delta,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ b, float eps,
                                                          const uint8_t* __restrict__ valid, long long M, int D,
                                                          int flags, float* __restrict__ x_out,
                                                          void* __restrict__ normed) {
  const int lane = threadIdx.x & 31;
  const long long warps_total = static_cast<long long>(gridDim.x) * kLnRowsPerBlock;
  for (long long row = static_cast<long long>(blockIdx.x) * kLnRowsPerBlock + (threadIdx.x >> 5); row < M;
       row += warps_total) {
  const int nchunk = D >> 3;
  const float* xr = x + row * D;
  bool row_valid = true;
  if (valid != nullptr) row_valid = valid[row] != 0;

  float v[NCH][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nchunk) {
      const float4 a0 = __ldcs(reinterpret_cast<const float4*>(xr) + 2 * c);
      const float4 a1 = __ldcs(reinterpret_cast<const float4*>(xr) + 2 * c + 1);
      v[i][0] = a0.x; v[i][1] = a0.y; v[i][2] = a0.z; v[i][3] = a0.w;
      v[i][4] = a1.x; v[i][5] = a1.y; v[i][6] = a1.z; v[i][7] = a1.w;
      if (delta != nullptr) {
        const uint4 dq = __ldcs(reinterpret_cast<const uint4*>(delta + row * D) + c);
        const __half2* dh = reinterpret_cast<const __half2*>(&dq);
        const bool keep = !(flags & TF_LN_MASK_DELTA) || row_valid;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(dh[j]);
          v[i][2 * j] += keep ? f.x : 0.f;
          v[i][2 * j + 1] += keep ? f.y : 0.f;
        }
      }
      if ((flags & TF_LN_MASK_X) && !row_valid) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[i][j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / static_cast<float>(D);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nchunk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        sq += d * d;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq / static_cast<float>(D) + eps);
  const bool zero_out = (flags & TF_LN_MASK_OUT) && !row_valid;

#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nchunk) {
      if (flags & TF_LN_WRITE_X) {
        float4* xo = reinterpret_cast<float4*>(x_out + row * D) + 2 * c;
        __stcs(xo, make_float4(v[i][0], v[i][1], v[i][2], v[i][3]));
        __stcs(xo + 1, make_float4(v[i][4], v[i][5], v[i][6], v[i][7]));
      }
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c + 1);
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(b) + 2 * c);
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(b) + 2 * c + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = zero_out ? 0.f : (v[i][j] - mean) * rstd * wv[j] + bv[j];
      if (flags & TF_LN_OUT_F32) {
        float4* no = reinterpret_cast<float4*>(static_cast<float*>(normed) + row * D) + 2 * c;
        __stcs(no, make_float4(y[0], y[1], y[2], y[3]));
        __stcs(no + 1, make_float4(y[4], y[5], y[6], y[7]));
      } else {
        uint4 q;
        q.x = pack_half2(y[0], y[1]);
        q.y = pack_half2(y[2], y[3]);
        q.z = pack_half2(y[4], y[5]);
        q.w = pack_half2(y[6], y[7]);
        reinterpret_cast<uint4*>(static_cast<__half*>(normed) + row * D)[c] = q;
      }
    }
  }
  }  // row loop
}

int ln_residual(const float* x, const void* delta, const float* w, const float* b, float eps,
                const uint8_t* valid, long long M, int D, int flags, float* x_out, void* normed,
                cudaStream_t stream) {
  if (M <= 0) return TF_OK;  // nothing to do
  if (D <= 0 || D % 8 != 0 || D > 4096)
    return set_error(TF_ERR_SHAPE, "ln_residual: D=%d must be a positive multiple of 8, <= 4096", D);
  if (!aligned16(x) || !aligned16(delta) || !aligned16(w) || !aligned16(b) || !aligned16(x_out) ||
      !aligned16(normed))
    return set_error(TF_ERR_ALIGN, "ln_residual: pointers must be 16-byte aligned");
  if (x == nullptr || w == nullptr || b == nullptr || normed == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_residual: x, w, b and normed are required");
  if ((flags & TF_LN_WRITE_X) && x_out == nullptr) return set_error(TF_ERR_SHAPE, "ln_residual: WRITE_X without x_out");
  if ((flags & (TF_LN_MASK_DELTA | TF_LN_MASK_X | TF_LN_MASK_OUT)) && valid == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_residual: mask flag without a valid-token mask");
  if (!(flags & (TF_LN_MASK_DELTA | TF_LN_MASK_X | TF_LN_MASK_OUT))) valid = nullptr;
  // grid-stride over rows with the device filled exactly (resident blocks
  // per SM from the occupancy of this instantiation)
  const int nch = (D / 8 + 31) / 32;
  const __half* dh = static_cast<const __half*>(delta);
  const long long need = (M + kLnRowsPerBlock - 1) / kLnRowsPerBlock;
#define TFB_LN_CASE(N)                                                                                        \
  {                                                                                                           \
    int per_sm = 1;                                                                                           \
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ln_residual_kernel<N>, 256, 0);                    \
    long long blocks = static_cast<long long>(device_sm_count()) * (per_sm > 0 ? per_sm : 1);                 \
    if (blocks > need) blocks = need;                                                                         \
    ln_residual_kernel<N><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, dh, w, b, eps, valid, M, D,   \
                                                                             flags, x_out, normed);           \
  }                                                                                                           \
  break;
  switch (nch <= 1 ? 1 : nch <= 2 ? 2 : nch <= 4 ? 4 : nch <= 8 ? 8 : 16) {
    case 1: TFB_LN_CASE(1)
    case 2: TFB_LN_CASE(2)
    case 4: TFB_LN_CASE(4)
    case 8: TFB_LN_CASE(8)
    default: TFB_LN_CASE(16)
  }
#undef TFB_LN_CASE
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "ln_residual launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
