// fp16 GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] = epilogue( A[M,K] · W[N,K]^T + bias[N] )      (all fp16 in HBM)
//
// This is the projection the reference runs four times per layer on its
// fp32-model fast path (packed QKV, out_proj, ffn_in+GELU, ffn_out:
// torch_transformer_benchmark.py:4138-4194, Triton kernel 1756-1803).
// Epilogues (all on the fp32 accumulator plus an fp32 bias):
//   EPI 0  C = fp16(acc + bias)
//   EPI 1  C = fp16(gelu_erf(acc + bias))        exact-erf GELU in fp32
//   EPI 2  x_out = mask_x(x_in + mask_delta(acc + bias))   fp32 residual
// EPI 2 is the residual add of the reference's next LayerNorm site
// (torch_transformer_benchmark.py:3988-3995) moved into the GEMM, with the
// same two masking points. Compared with the reference's fp16 fast path this
// drops three fp16 roundings (bias, GELU input, residual delta); the result
// is closer to the fp32 eager model the accuracy gate compares against.
//
// Optional split weights (a_repeat = 2): W holds [W_hi | W_lo] along K, with
// W_lo = fp16(W - W_hi), and A is streamed twice, so the product sees the
// fp32 weight to ~2^-22 at twice the tensor-core work.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A and W tiles (128B-swizzled) into a STAGES ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, bias/GELU, stores
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle row of fp16
constexpr int kGemmThreads = 192;

struct GemmArgs {
  const float* bias;
  __half* C;  // EPI 0/1
  long long ldc;
  const float* x_in;  // EPI 2
  float* x_out;
  long long ldx;
  const uint8_t* valid;
  int mask_mode;  // EPI 2: 0 none, 1 mask_delta, 2 mask_x
  int M, N, K;    // K: columns of A
  int a_repeat;   // 1, or 2 for split weights (W has a_repeat*K columns)
  int m_tiles, n_tiles;
  int* status;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, tmem slot
  static constexpr int kBytes = kBarOffset + (2 * STAGES + 5) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     GemmArgs p) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int total_tiles = p.m_tiles * p.n_tiles;
  const int a_blocks = (p.K + kGemmBK - 1) / kGemmBK;
  const int k_blocks = a_blocks * p.a_repeat;

  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.n_tiles) * kGemmBM;
        const int n0 = (t % p.n_tiles) * BN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * L::kStageBytes;
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          const int akb = kb < a_blocks ? kb : kb - a_blocks;
          tma_load_2d(sa, &tmA, &full[s], akb * kGemmBK, m0);
          // W block: columns [kb*64, kb*64+64) of [W_hi | W_lo]; with a
          // K tail the lo half starts at column K, not at a_blocks*64
          const int wcol = kb < a_blocks ? kb * kGemmBK : p.K + akb * kGemmBK;
          tma_load_2d(sa + L::kABytes, &tmB, &full[s], wcol, n0);
        }
      }
      // Drain: every load this thread issued must land before the CTA exits.
      const int first = it > STAGES ? it - STAGES : 0;
      for (int j = first; j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_f16_f32(kGemmBM, BN);
      const uint32_t smem_base = smem_u32(smem);
      int it = 0;
      int tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++tc) {
        const int a = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + s * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sb + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[a]);
      }
      // Drain: all MMAs issued above complete before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, kDevTimeoutDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int tc = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tc) {
      const int m0 = (t / p.n_tiles) * kGemmBM;
      const int n0 = (t % p.n_tiles) * BN;
      const int a = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      if (!mbar_wait(&tfull[a], aph, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_addr + c * 32, r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          // accumulator fully read: hand the buffer back to the MMA warp
          tc_fence_before();
          mbar_arrive(&tempty[a]);
        }
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.N) continue;
        const float4* bsrc = reinterpret_cast<const float4*>(p.bias + col0);
        float acc[32];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 bq = __ldg(bsrc + v);
          acc[4 * v + 0] = __uint_as_float(r[4 * v + 0]) + bq.x;
          acc[4 * v + 1] = __uint_as_float(r[4 * v + 1]) + bq.y;
          acc[4 * v + 2] = __uint_as_float(r[4 * v + 2]) + bq.z;
          acc[4 * v + 3] = __uint_as_float(r[4 * v + 3]) + bq.w;
        }
        if constexpr (EPI == 2) {
          const long long xoff = static_cast<long long>(row) * p.ldx + col0;
          const float4* xi = reinterpret_cast<const float4*>(p.x_in + xoff);
          float4* xo = reinterpret_cast<float4*>(p.x_out + xoff);
          bool valid = true;
          if (p.mask_mode != 0) valid = p.valid[row] != 0;
          const float dscale = (p.mask_mode == 1 && !valid) ? 0.f : 1.f;
          const bool zero = p.mask_mode == 2 && !valid;
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float4 xv = xi[v];
            float4 o;
            o.x = zero ? 0.f : xv.x + acc[4 * v + 0] * dscale;
            o.y = zero ? 0.f : xv.y + acc[4 * v + 1] * dscale;
            o.z = zero ? 0.f : xv.z + acc[4 * v + 2] * dscale;
            o.w = zero ? 0.f : xv.w + acc[4 * v + 3] * dscale;
            xo[v] = o;
          }
        } else {
          uint32_t outw[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float h0 = acc[2 * j], h1 = acc[2 * j + 1];
            if constexpr (EPI == 1) {
              h0 = h0 * 0.5f * (1.0f + erff(h0 * 0.7071067811865476f));
              h1 = h1 * 0.5f * (1.0f + erff(h1 * 0.7071067811865476f));
            }
            outw[j] = pack_half2(h0, h1);
          }
          __half* crow = p.C + static_cast<long long>(row) * p.ldc + col0;
          uint4* dst = reinterpret_cast<uint4*>(crow);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(outw[4 * v], outw[4 * v + 1], outw[4 * v + 2], outw[4 * v + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int BN, int STAGES, int EPI>
static int launch_gemm_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                           cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_f16_tcgen05<BN, STAGES, EPI>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(gemm): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  kern<<<grid, kGemmThreads, L::kAlloc, stream>>>(ta, tb, args);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "gemm launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

// Pick the N tile: 256 unless 128 finishes the grid in fewer weighted waves
// (a 128-wide tile does half the work per tile at ~10% lower efficiency).
static int choose_bn(int m_tiles, int N, int sms) {
  if (N % 256 != 0 && N % 128 != 0) return 64;
  const long long t256 = (N % 256 == 0) ? (long long)m_tiles * (N / 256) : -1;
  const long long t128 = (long long)m_tiles * (N / 128);
  if (t256 < 0) return 128;
  const double w256 = 2.0 * double((t256 + sms - 1) / sms);
  const double w128 = 1.1 * double((t128 + sms - 1) / sms);
  if (t128 < sms / 2) {
    // very few tiles: spread the weight reads over more SMs
    const long long t64 = (long long)m_tiles * (N / 64);
    if (t64 <= sms) return 64;
  }
  return (w128 < w256) ? 128 : 256;
}

int gemm_f16(const GemmCall& g, cudaStream_t stream) {
  const long long M = g.M, N = g.N, K = g.K;
  if (M <= 0 || N <= 0 || K <= 0) return set_error(TF_ERR_SHAPE, "gemm: empty shape M=%lld N=%lld K=%lld", M, N, K);
  if (M > (1ll << 31) - 1 || N > 65535ll * 64 || K > (1 << 24))
    return set_error(TF_ERR_SHAPE, "gemm: shape out of range");
  if (N % 32 != 0) return set_error(TF_ERR_SHAPE, "gemm: N=%lld must be a multiple of 32", N);
  if (g.a_repeat != 1 && g.a_repeat != 2) return set_error(TF_ERR_SHAPE, "gemm: a_repeat must be 1 or 2");
  if (K % 8 != 0 || g.lda % 8 != 0 || g.ldw % 8 != 0)
    return set_error(TF_ERR_ALIGN, "gemm: K and leading dimensions must be multiples of 8 elements");
  if (g.lda < K || g.ldw < K * g.a_repeat) return set_error(TF_ERR_SHAPE, "gemm: leading dimension smaller than row");
  if (!aligned16(g.A) || !aligned16(g.W) || !aligned16(g.bias) || g.A == nullptr || g.W == nullptr ||
      g.bias == nullptr)
    return set_error(TF_ERR_ALIGN, "gemm: A, W and bias must be non-null and 16-byte aligned");
  if (g.epilogue == 0 || g.epilogue == 1) {
    if (g.C == nullptr || !aligned16(g.C) || g.ldc % 8 != 0 || g.ldc < N)
      return set_error(TF_ERR_ALIGN, "gemm: C must be 16-byte aligned with a pitch >= N, multiple of 8");
  } else if (g.epilogue == 2) {
    if (g.x_in == nullptr || g.x_out == nullptr || !aligned16(g.x_in) || !aligned16(g.x_out) || g.ldx % 4 != 0 ||
        g.ldx < N)
      return set_error(TF_ERR_ALIGN, "gemm: residual x must be 16-byte aligned with a pitch >= N, multiple of 4");
    if (g.mask_mode < 0 || g.mask_mode > 2) return set_error(TF_ERR_SHAPE, "gemm: mask mode %d", g.mask_mode);
    if (g.mask_mode != 0 && g.valid == nullptr) return set_error(TF_ERR_SHAPE, "gemm: mask without valid rows");
  } else {
    return set_error(TF_ERR_SHAPE, "gemm: unknown epilogue %d", g.epilogue);
  }

  const int sms = device_sm_count();
  const int m_tiles = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  int bn = g.tile_n > 0 ? g.tile_n : choose_bn(m_tiles, static_cast<int>(N), sms);
  if (N % bn != 0) bn = (N % 128 == 0) ? 128 : 64;

  CUtensorMap ta, tb;
  int rc = make_tmap_2d_f16(&ta, g.A, K, M, g.lda, kGemmBK, kGemmBM);
  if (rc) return rc;
  rc = make_tmap_2d_f16(&tb, g.W, K * g.a_repeat, N, g.ldw, kGemmBK, bn);
  if (rc) return rc;

  GemmArgs args;
  args.bias = g.bias;
  args.C = static_cast<__half*>(g.C);
  args.ldc = g.ldc;
  args.x_in = g.x_in;
  args.x_out = g.x_out;
  args.ldx = g.ldx;
  args.valid = g.valid;
  args.mask_mode = g.epilogue == 2 ? g.mask_mode : 0;
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.a_repeat = g.a_repeat;
  args.m_tiles = m_tiles;
  args.n_tiles = static_cast<int>((N + bn - 1) / bn);
  args.status = device_status_ptr();
  if (args.status == nullptr) return last_error_code();
  const long long tiles = static_cast<long long>(args.m_tiles) * args.n_tiles;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);

#define TFB_GEMM_EPI(BN, ST)                                                         \
  switch (g.epilogue) {                                                              \
    case 0: return launch_gemm_cfg<BN, ST, 0>(ta, tb, args, grid, stream);           \
    case 1: return launch_gemm_cfg<BN, ST, 1>(ta, tb, args, grid, stream);           \
    default: return launch_gemm_cfg<BN, ST, 2>(ta, tb, args, grid, stream);          \
  }
  if (bn == 256) {
    TFB_GEMM_EPI(256, 4)
  } else if (bn == 128) {
    TFB_GEMM_EPI(128, 6)
  }
  TFB_GEMM_EPI(64, 8)
#undef TFB_GEMM_EPI
}

}  // namespace tfb
