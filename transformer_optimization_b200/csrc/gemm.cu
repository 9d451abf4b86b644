// fp16 GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] = epilogue( A[M,K] · W[N,K]^T + bias[N] )      (all fp16 in HBM)
//
// This is the projection the reference runs four times per layer on its
// fp32-model fast path (packed QKV, out_proj, ffn_in+GELU, ffn_out:
// torch_transformer_benchmark.py:4138-4194, Triton kernel 1756-1803). The
// epilogue keeps the reference's rounding order exactly: bias is added to the
// fp32 accumulator, the sum is rounded to fp16, and only then (for ffn_in)
// the exact-erf GELU runs in fp32 on the rounded value and is rounded again
// (torch_transformer_benchmark.py:1795-1802).
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
  const __half* bias;
  __half* C;
  int M, N, K;
  long long ldc;
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
  const int k_blocks = (p.K + kGemmBK - 1) / kGemmBK;

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
          tma_load_2d(sa, &tmA, &full[s], kb * kGemmBK, m0);
          tma_load_2d(sa + L::kABytes, &tmB, &full[s], kb * kGemmBK, n0);
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
      __half* crow = p.C + static_cast<long long>(row) * p.ldc + n0;
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
        const uint4* bsrc = reinterpret_cast<const uint4*>(p.bias + col0);
        uint32_t outw[16];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 bq = __ldg(bsrc + v);
          const __half2* bh = reinterpret_cast<const __half2*>(&bq);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 bf = __half22float2(bh[j]);
            float h0 = __half2float(__float2half_rn(__uint_as_float(r[v * 8 + 2 * j]) + bf.x));
            float h1 = __half2float(__float2half_rn(__uint_as_float(r[v * 8 + 2 * j + 1]) + bf.y));
            if (EPI == 1) {
              h0 = h0 * 0.5f * (1.0f + erff(h0 * 0.7071067811865476f));
              h1 = h1 * 0.5f * (1.0f + erff(h1 * 0.7071067811865476f));
            }
            outw[v * 4 + j] = pack_half2(h0, h1);
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) dst[v] = make_uint4(outw[4 * v], outw[4 * v + 1], outw[4 * v + 2], outw[4 * v + 3]);
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

int gemm_f16(const void* A, long long lda, const void* W, long long ldw, const void* bias, void* C,
             long long ldc, long long M, long long N, long long K, int epilogue, int force_bn,
             cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(TF_ERR_SHAPE, "gemm: empty shape M=%lld N=%lld K=%lld", M, N, K);
  if (M > (1ll << 31) - 1 || N > 65535 * 64 || K > (1 << 24))
    return set_error(TF_ERR_SHAPE, "gemm: shape out of range");
  if (N % 32 != 0) return set_error(TF_ERR_SHAPE, "gemm: N=%lld must be a multiple of 32", N);
  if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0 || ldc % 8 != 0)
    return set_error(TF_ERR_ALIGN, "gemm: K and leading dimensions must be multiples of 8 elements");
  if (lda < K || ldw < K || ldc < N) return set_error(TF_ERR_SHAPE, "gemm: leading dimension smaller than row");
  if (!aligned16(A) || !aligned16(W) || !aligned16(C) || !aligned16(bias))
    return set_error(TF_ERR_ALIGN, "gemm: A, W, bias and C must be 16-byte aligned");
  if (epilogue != 0 && epilogue != 1) return set_error(TF_ERR_SHAPE, "gemm: unknown epilogue %d", epilogue);

  const int sms = device_sm_count();
  const int m_tiles = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  int bn = force_bn > 0 ? force_bn : choose_bn(m_tiles, static_cast<int>(N), sms);
  if (N % bn != 0) bn = (N % 128 == 0) ? 128 : 64;
  if (N % bn != 0) bn = 32;
  if (bn == 32) bn = 64;  // smallest tile; the epilogue guards the column tail

  CUtensorMap ta, tb;
  int rc = make_tmap_2d_f16(&ta, A, K, M, lda, kGemmBK, kGemmBM);
  if (rc) return rc;
  rc = make_tmap_2d_f16(&tb, W, K, N, ldw, kGemmBK, bn);
  if (rc) return rc;

  GemmArgs args;
  args.bias = static_cast<const __half*>(bias);
  args.C = static_cast<__half*>(C);
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.ldc = ldc;
  args.m_tiles = m_tiles;
  args.n_tiles = static_cast<int>((N + bn - 1) / bn);
  args.status = device_status_ptr();
  if (args.status == nullptr) return last_error_code();
  const long long tiles = static_cast<long long>(args.m_tiles) * args.n_tiles;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);

  if (bn == 256) {
    return epilogue ? launch_gemm_cfg<256, 4, 1>(ta, tb, args, grid, stream)
                    : launch_gemm_cfg<256, 4, 0>(ta, tb, args, grid, stream);
  } else if (bn == 128) {
    return epilogue ? launch_gemm_cfg<128, 6, 1>(ta, tb, args, grid, stream)
                    : launch_gemm_cfg<128, 6, 0>(ta, tb, args, grid, stream);
  }
  return epilogue ? launch_gemm_cfg<64, 8, 1>(ta, tb, args, grid, stream)
                  : launch_gemm_cfg<64, 8, 0>(ta, tb, args, grid, stream);
}

}  // namespace tfb
