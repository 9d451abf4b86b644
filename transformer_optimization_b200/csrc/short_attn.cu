// Attention of short sequences (S <= 128 tokens, head_dim 64) in one CTA
// per (batch element, head), for the few-row forwards (BASELINE's c1: S = 128,
// c2: S = 64) where the general flash kernel's pipeline is mostly set-up.
//
//   out[b, i, h*64 : h*64+64] = sum_j softmax_j(scale * q_i . k_j) v_j
//
// Replaces the reference's short-sequence attention (_short_attn_kernel and
// _triton_short_attention, torch_transformer_benchmark.py:1193-1304,
// 1596-1625) on the fp32 model's fp16 path. The q, k, v of the head come
// either from packed fp16 q|k|v rows or, to save the launch of a reduce
// kernel, straight from the fp32 split-K partial sums of the QKV projection
// (summed here in split order, plus the bias, rounded to fp16 once: the same
// values the split-K reduce would have stored). All 256 threads stage the
// three 128 x 64 fp16 tiles in shared memory in the 128-byte-swizzled
// K-major layout of the tensor-core operands (rows past the sequence are
// zero); then one thread issues S = Q K^T (tcgen05, fp32 in TMEM), warps
// 4..7 run the softmax one query row per thread (keys past the sequence, above
// the causal diagonal or marked invalid are masked; exp2 with the scale folded
// into log2(e); P rounded to fp16 into TMEM over S), the same thread issues
// O = P V with P read from TMEM, and warps 4..7 store O / l. A row whose keys
// are all masked gets 0. Every wait is bounded (common.cuh).
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kSaThreads = 256;
constexpr int kSaTile = 128 * 64 * 2;  // one 128-row x 64-column fp16 tile
constexpr int kSaQ = 0;
constexpr int kSaK = kSaTile;
constexpr int kSaV = 2 * kSaTile;
constexpr int kSaBarOff = 3 * kSaTile;  // s_full, p_full, o_full, drain
constexpr int kSaSmem = kSaBarOff + 4 * 8 + 16 + 1024;
constexpr uint32_t kSaTmemCols = 256;  // S / P at [0, 128), O at [128, 192)
constexpr uint32_t kSaTmemO = 128;

struct SaParams {
  const float* part;
  const float* bias;
  const uint16_t* qkv;
  const uint8_t* key_valid;
  uint16_t* out;
  long long ld_o;
  long long plane;  // rows * 3D: one split's partials
  int splits;
  int seq, d_model, causal;
  float scale_log2;
  int* status;
};

// Element (row, col) of a 128-byte-swizzled K-major 64-column fp16 tile:
// byte row * 128 + ((col / 8) ^ (row % 8)) * 16 + (col % 8) * 2.
__device__ __forceinline__ uint32_t sa_chunk_offset(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) * 16));
}

__global__ void __launch_bounds__(kSaThreads, 1) short_attn_kernel(const SaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSaBarOff);
  uint64_t* s_full = bars;
  uint64_t* p_full = bars + 1;
  uint64_t* o_full = bars + 2;
  uint64_t* drain = bars + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int warp = warp_id();
  const int lane = lane_id();
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  if (threadIdx.x == 0) {
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kSaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  // ---- stage Q, K, V (3 tiles x 128 rows x 8 chunks of 8 columns) ----
  const long long row0 = static_cast<long long>(b) * p.seq;
  const int ld = 3 * p.d_model;
#pragma unroll 2
  for (int c = threadIdx.x; c < 3 * 128 * 8; c += kSaThreads) {
    const int which = c >> 10;  // 0 q, 1 k, 2 v
    const int row = (c >> 3) & 127;
    const int chunk = c & 7;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < p.seq) {
      const long long col = static_cast<long long>(which) * p.d_model + h * 64 + chunk * 8;
      const long long off = (row0 + row) * ld + col;
      if (p.part != nullptr) {
        float4 a0 = *reinterpret_cast<const float4*>(p.part + off);
        float4 a1 = *reinterpret_cast<const float4*>(p.part + off + 4);
        for (int s = 1; s < p.splits; ++s) {
          const float4 q0 = *reinterpret_cast<const float4*>(p.part + s * p.plane + off);
          const float4 q1 = *reinterpret_cast<const float4*>(p.part + s * p.plane + off + 4);
          a0.x += q0.x; a0.y += q0.y; a0.z += q0.z; a0.w += q0.w;
          a1.x += q1.x; a1.y += q1.y; a1.z += q1.z; a1.w += q1.w;
        }
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias + col));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias + col + 4));
        v = make_uint4(pack_half2(a0.x + b0.x, a0.y + b0.y), pack_half2(a0.z + b0.z, a0.w + b0.w),
                       pack_half2(a1.x + b1.x, a1.y + b1.y), pack_half2(a1.z + b1.z, a1.w + b1.w));
      } else {
        v = *reinterpret_cast<const uint4*>(p.qkv + off);
      }
    }
    *reinterpret_cast<uint4*>(smem + which * kSaTile + sa_chunk_offset(row, chunk)) = v;
  }
  fence_proxy_async_smem();  // the tensor core reads the tiles through the async proxy
  __syncthreads();

  bool ok = true;
  if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t base = smem_u32(smem);
      constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, 64, false, true);  // K-major P, MN-major V
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16_ss(tmem, smem_desc_sw128(base + kSaQ + k * 32, 16, 1024),
                    smem_desc_sw128(base + kSaK + k * 32, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
      umma_commit(s_full);
      if (mbar_wait(p_full, 0, p.status, kDevTimeoutMma)) {
        tc_fence_after();
        // P: 128 keys = 64 TMEM columns, 8 per MMA; V MN-major, 16 keys = 2048 B
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ts(tmem + kSaTmemO, tmem + k * 8, smem_desc_sw128(base + kSaV + k * 2048, 16384, 1024), idesc_o,
                      k > 0 ? 1u : 0u);
      }
      umma_commit(o_full);
      umma_commit(drain);  // every MMA of this thread completes before TMEM is released
      mbar_wait(drain, 0, p.status, kDevTimeoutDrain);
    }
  } else if (warp >= 4) {
    // ---------------- softmax and output (one query row per thread) ----------------
    const int qtr = warp & 3;
    const int r = qtr * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
    float l = 0.f;
    ok = mbar_wait(s_full, 0, p.status, kDevTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      float s[128];
      {
        uint32_t v[128];
        tmem_ld128(tmem + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(v[i]);
      }
      const int lim = p.causal ? (r + 1 < p.seq ? r + 1 : p.seq) : p.seq;
      const uint8_t* kv = p.key_valid != nullptr ? p.key_valid + row0 : nullptr;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        bool keep = i < lim;
        if (kv != nullptr && keep) keep = kv[i] != 0;
        s[i] = keep ? s[i] : -INFINITY;
        mx = fmaxf(mx, s[i]);
      }
      const float c = p.scale_log2;
      const float m = mx == -INFINITY ? 0.f : mx * c;
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float e0 = exp2f(fmaf(s[2 * i], c, -m));
        const float e1 = exp2f(fmaf(s[2 * i + 1], c, -m));
        l += e0 + e1;
        pk[i] = pack_half2(e0, e1);
      }
      tmem_st64(tmem + lane_off, pk);
      tmem_wait_st_all();
    }
    tc_fence_before();
    mbar_arrive(p_full);  // also after a failed wait: the MMA thread's wait then ends
    if (ok && mbar_wait(o_full, 0, p.status, kDevTimeoutSoftmax)) {
      tc_fence_after();
      uint32_t ov[64];
      tmem_ld64(tmem + lane_off + kSaTmemO, ov);
      tmem_wait_ld();
      if (r < p.seq) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.out + (row0 + r) * p.ld_o + h * 64);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = make_uint4(pack_half2(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv),
                              pack_half2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv),
                              pack_half2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv),
                              pack_half2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kSaTmemCols);
  }
}

int short_attention(const ShortAttnArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.heads <= 0 || a.seq <= 0) return TF_OK;
  if (a.head_dim != 64) return set_error(TF_ERR_SHAPE, "short attention: head_dim=%lld (64 supported)", a.head_dim);
  if (a.seq > 128) return set_error(TF_ERR_SHAPE, "short attention: seq=%lld (at most 128)", a.seq);
  if (a.batch > 65535 || a.heads > 65535) return set_error(TF_ERR_SHAPE, "short attention: sizes out of range");
  if ((a.part == nullptr) == (a.qkv == nullptr))
    return set_error(TF_ERR_SHAPE, "short attention: exactly one of the partials and the packed q|k|v");
  if (a.part != nullptr && (a.bias == nullptr || a.splits < 1 || !aligned16(a.part) || !aligned16(a.bias)))
    return set_error(TF_ERR_ALIGN, "short attention: partials and bias 16-byte aligned, splits >= 1");
  if (a.qkv != nullptr && !aligned16(a.qkv)) return set_error(TF_ERR_ALIGN, "short attention: q|k|v 16-byte aligned");
  if (a.out == nullptr || !aligned16(a.out) || a.ld_o % 8 != 0 || a.ld_o < a.heads * 64)
    return set_error(TF_ERR_ALIGN, "short attention: out 16-byte aligned with a pitch >= heads*64, multiple of 8");
  if (a.flags & ~TF_ATTN_CAUSAL) return set_error(TF_ERR_SHAPE, "short attention: flags %d (TF_ATTN_CAUSAL)", a.flags);
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(short_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSaSmem);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(short attention): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  SaParams p;
  p.part = a.part;
  p.bias = a.bias;
  p.qkv = static_cast<const uint16_t*>(a.qkv);
  p.key_valid = a.key_valid;
  p.out = static_cast<uint16_t*>(a.out);
  p.ld_o = a.ld_o;
  p.plane = a.batch * a.seq * 3 * a.heads * 64;
  p.splits = a.splits;
  p.seq = static_cast<int>(a.seq);
  p.d_model = static_cast<int>(a.heads * 64);
  p.causal = (a.flags & TF_ATTN_CAUSAL) ? 1 : 0;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = device_status_ptr();
  if (p.status == nullptr) return last_error_code();
  cudaError_t e = launch_k(short_attn_kernel, dim3(static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch)),
                           dim3(kSaThreads), kSaSmem, stream, p);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "short attention launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
