// Flash attention forward on the 5th-generation tensor cores.
//
//   out_i = sum_j softmax_j(scale * q_i . k_j) v_j       (fp16 in, fp32 math)
//
// Replaces the attention of the reference's fp32-model fast path
// (F.scaled_dot_product_attention / _short_attn_kernel / _flash_attn_kernel,
// torch_transformer_benchmark.py:4146-4161, 1193-1418). Like the reference's
// flash kernel it never materialises the score matrix: scores live in TMEM,
// probabilities in shared memory, one 128-key block at a time, with the
// online-softmax running max / sum (m, l) per query row and exp2 with the
// scale folded into log2(e) (torch_transformer_benchmark.py:1427-1428).
//
// One CTA = one 128-query tile of one (batch, head); 192 threads:
//   warp 0      TMA producer: the Q tile once, then K_j / V_j blocks
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T          -> TMEM S[j%2]   (fp32, 128 cols)
//                 O_j = P_j V_j          -> TMEM O[j%2]   (fp32, hd cols)
//   warps 2..5  softmax + correction: thread t owns query row t. It reads
//               S_j from TMEM, writes P_j (fp16, 128B-swizzled K-major) to
//               shared memory, and folds O_j into its fp32 register
//               accumulator with the running-max rescale.
// S_{j+1} is issued while the softmax warps work on S_j (two S buffers), so
// the tensor core and the softmax overlap.
//
// The kernel also emits the natural-log sum-exp per row, used to merge the
// partial results of context-parallel ring attention exactly.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kAttnBM = 128;  // query rows per CTA
constexpr int kAttnBN = 128;  // keys per block
constexpr int kAttnThreads = 192;

struct AttnKParams {
  void* out;
  long long ld_o, bs_o;
  float* lse;
  const uint8_t* key_valid;
  int heads, seq_q, seq_k;
  int q_tiles;
  float scale_log2;  // scale * log2(e)
  long long q_pos0, k_pos0;
  int flags;
  int* status;
};

template <int HD>
struct AttnSmem {
  static constexpr int kQBytes = kAttnBM * HD * 2;
  static constexpr int kKBytes = kAttnBN * HD * 2;
  static constexpr int kStages = HD == 64 ? 3 : 2;
  static constexpr int kStageBytes = 2 * kKBytes;  // K then V
  static constexpr int kPBytes = kAttnBM * kAttnBN * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = kQOff + kQBytes;
  static constexpr int kPOff = kKVOff + kStages * kStageBytes;
  static constexpr int kBarOff = kPOff + 2 * kPBytes;
  // q_full, kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2],
  // p_free[2], o_full[2], o_free[2], drain, + tmem slot
  static constexpr int kNumBars = 1 + 2 * kStages + 12 + 1;
  static constexpr int kBytes = kBarOff + kNumBars * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ float fmax3(float a, float b) { return fmaxf(a, b); }

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_fwd_tcgen05(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, AttnKParams p) {
  using L = AttnSmem<HD>;
  constexpr int ST = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* p_free = p_full + 2;
  uint64_t* o_full = p_free + 2;
  uint64_t* o_free = o_full + 2;
  uint64_t* drain = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  // longest (causal) tiles first
  const int q_tile = p.q_tiles - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = q_tile * kAttnBM;

  // number of key blocks this tile needs
  long long k_end = p.seq_k;
  if (p.flags & TF_ATTN_CAUSAL) {
    const long long last_q = p.q_pos0 + q0 + kAttnBM - 1;  // global position of the tile's last row
    const long long lim = last_q - p.k_pos0 + 1;           // keys [0, lim) can be admissible
    if (lim < k_end) k_end = lim;
  }
  const int n_blocks = k_end <= 0 ? 0 : static_cast<int>((k_end + kAttnBN - 1) / kAttnBN);

  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmQ);
    tma_prefetch_map(&tmK);
    tma_prefetch_map(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM columns: S[0] 0..127, S[1] 128..255, O[0] 256.., O[1] 256+HD..
  const uint32_t tm_s0 = tmem_base;
  const uint32_t tm_o0 = tmem_base + 256;

  if (warp == 0) {
    if (lane == 0 && n_blocks > 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(q_full, L::kQBytes);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_3d(smem + L::kQOff + c * (kAttnBM * 128), &tmQ, q_full, h * HD + c * 64, q0, b);
      int j = 0;
      for (; j < n_blocks; ++j) {
        const int s = j % ST;
        const uint32_t ph = (j / ST) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1, p.status, kDevTimeoutProducer)) break;
        uint8_t* kdst = smem + L::kKVOff + s * L::kStageBytes;
        uint8_t* vdst = kdst + L::kKBytes;
        mbar_arrive_expect_tx(&kv_full[s], L::kStageBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_3d(kdst + c * (kAttnBN * 128), &tmK, &kv_full[s], h * HD + c * 64, j * kAttnBN, b);
          tma_load_3d(vdst + c * (kAttnBN * 128), &tmV, &kv_full[s], h * HD + c * 64, j * kAttnBN, b);
        }
      }
      // drain the loads issued above
      mbar_wait(q_full, 0, p.status, kDevTimeoutDrain);
      const int first = j > ST ? j - ST : 0;
      for (int i = first; i < j; ++i) mbar_wait(&kv_full[i % ST], (i / ST) & 1, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_blocks > 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = idesc_f16_f32(kAttnBM, kAttnBN);             // K-major Q, K-major K
      constexpr uint32_t idesc_o = idesc_f16_f32(kAttnBM, HD, false, true);     // K-major P, MN-major V
      const uint32_t sq = smem_u32(smem + L::kQOff);
      const uint32_t skv = smem_u32(smem + L::kKVOff);
      const uint32_t sp = smem_u32(smem + L::kPOff);
      bool ok = mbar_wait(q_full, 0, p.status, kDevTimeoutMma);
      auto issue_s = [&](int j) -> bool {
        const int s = j % ST;
        if (!mbar_wait(&kv_full[s], (j / ST) & 1, p.status, kDevTimeoutMma)) return false;
        if (!mbar_wait(&s_free[j & 1], ((j >> 1) & 1) ^ 1, p.status, kDevTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t kb = skv + s * L::kStageBytes;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * (kAttnBM * 128) + (k & 3) * 32;
          const uint64_t ad = smem_desc_sw128(sq + off, 16, 1024);
          const uint64_t bd = smem_desc_sw128(kb + (k >> 2) * (kAttnBN * 128) + (k & 3) * 32, 16, 1024);
          umma_f16_ss(tm_s0 + (j & 1) * 128, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_blocks && ok; ++j) {
        if (j + 1 < n_blocks) {
          if (!(ok = issue_s(j + 1))) break;
        }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status, kDevTimeoutMma)) break;
        if (!mbar_wait(&o_free[j & 1], ((j >> 1) & 1) ^ 1, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const int s = j % ST;
        const uint32_t vb = skv + s * L::kStageBytes + L::kKBytes;
        const uint32_t pb = sp + (j & 1) * L::kPBytes;
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k) {
          // P: K-major, 64-key column blocks of 16 KB; V: MN-major, 8-key
          // groups at 1024 B (SBO), 64-wide head-dim blocks at 16 KB (LBO).
          const uint64_t ad = smem_desc_sw128(pb + (k >> 2) * (kAttnBM * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(vb + k * 2048, kAttnBN * 128, 1024);
          umma_f16_ss(tm_o0 + (j & 1) * HD, ad, bd, idesc_o, k > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[j & 1]);
        umma_commit(&kv_empty[s]);
        umma_commit(&p_free[j & 1]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, kDevTimeoutDrain);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 2..5) -------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const long long q_glob = p.q_pos0 + q0 + r;
    const bool causal = (p.flags & TF_ATTN_CAUSAL) != 0;
    const uint8_t* kvalid = p.key_valid ? p.key_valid + static_cast<long long>(b) * p.seq_k : nullptr;
    uint8_t* pbase = smem + L::kPOff;

    float o_acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o_acc[i] = 0.f;
    float m2 = -INFINITY;  // running max in the scaled log2 domain
    float l = 0.f;
    float alpha_prev = 0.f;
    bool ok = true;

    auto fold = [&](int jb, float alpha) -> bool {
      if (!mbar_wait(&o_full[jb & 1], (jb >> 1) & 1, p.status, kDevTimeoutSoftmax)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tm_o0 + lane_off + (jb & 1) * HD + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o_acc[c * 32 + i] = o_acc[c * 32 + i] * alpha + __uint_as_float(v[i]);
      }
      tc_fence_before();
      mbar_arrive(&o_free[jb & 1]);
      return true;
    };

    for (int j = 0; j < n_blocks; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.status, kDevTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tm_s0 + lane_off + (j & 1) * 128;
      const long long kbase = static_cast<long long>(j) * kAttnBN;
      // keys of this block that need masking at all
      const bool need_mask = kvalid != nullptr || kbase + kAttnBN > p.seq_k ||
                             (causal && p.k_pos0 + kbase + kAttnBN - 1 > p.q_pos0 + q0);
      // pass 1: row max
      float mj = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(s_addr + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float t = __uint_as_float(v[i]) * p.scale_log2;
          if (need_mask) {
            const long long kk = kbase + c * 32 + i;
            bool bad = kk >= p.seq_k;
            if (causal) bad |= (p.k_pos0 + kk > q_glob);
            if (kvalid != nullptr && !bad) bad |= kvalid[kk] == 0;
            t = bad ? -INFINITY : t;
          }
          mj = fmaxf(mj, t);
        }
      }
      const float m_new = fmaxf(m2, mj);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = (m2 == -INFINITY) ? 0.f : exp2f(m2 - m_use);
      // P buffer j%2 must be free (PV of block j-2 done)
      if (!mbar_wait(&p_free[j & 1], ((j >> 1) & 1) ^ 1, p.status, kDevTimeoutSoftmax)) {
        ok = false;
        break;
      }
      // pass 2: probabilities -> fp16 -> swizzled shared memory, row sum
      float rs = 0.f;
      uint8_t* prow = pbase + (j & 1) * L::kPBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(s_addr + c * 32, v);
        tmem_wait_ld();
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float t0 = __uint_as_float(v[i]) * p.scale_log2;
          float t1 = __uint_as_float(v[i + 1]) * p.scale_log2;
          if (need_mask) {
            const long long k0 = kbase + c * 32 + i;
            bool bad0 = k0 >= p.seq_k, bad1 = k0 + 1 >= p.seq_k;
            if (causal) {
              bad0 |= (p.k_pos0 + k0 > q_glob);
              bad1 |= (p.k_pos0 + k0 + 1 > q_glob);
            }
            if (kvalid != nullptr) {
              if (!bad0) bad0 |= kvalid[k0] == 0;
              if (!bad1) bad1 |= kvalid[k0 + 1] == 0;
            }
            t0 = bad0 ? -INFINITY : t0;
            t1 = bad1 ? -INFINITY : t1;
          }
          const __half2 ph = __floats2half2_rn(exp2f(t0 - m_use), exp2f(t1 - m_use));
          const float2 pf = __half22float2(ph);
          rs += pf.x + pf.y;
          packed[i >> 1] = *reinterpret_cast<const uint32_t*>(&ph);
        }
        // 32 keys = 4 chunks of 16 B; chunk index within the 64-key block
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = c * 4 + q;       // 0..15 over the 128 keys
          const int blk = chunk >> 3;        // 64-key column block
          const int cc = (chunk & 7) ^ (r & 7);
          *reinterpret_cast<uint4*>(prow + blk * (kAttnBM * 128) + cc * 16) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[j & 1]);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[j & 1]);
      l = l * alpha + rs;
      m2 = m_new;
      if (j >= 1) {
        if (!fold(j - 1, alpha_prev)) {
          ok = false;
          break;
        }
      }
      alpha_prev = alpha;
    }
    if (ok && n_blocks > 0) ok = fold(n_blocks - 1, alpha_prev);

    // ---------------- epilogue ----------------
    const int row = q0 + r;
    if (ok && row < p.seq_q) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      if (p.lse != nullptr) {
        const float lse = l > 0.f ? (m2 + __log2f(l)) * 0.69314718055994531f : -INFINITY;
        p.lse[(static_cast<long long>(b) * p.heads + h) * p.seq_q + row] = lse;
      }
      const long long obase = static_cast<long long>(b) * p.bs_o + static_cast<long long>(row) * p.ld_o + h * HD;
      if (p.flags & TF_ATTN_OUT_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase);
#pragma unroll
        for (int i = 0; i < HD / 4; ++i)
          dst[i] = make_float4(o_acc[4 * i] * inv, o_acc[4 * i + 1] * inv, o_acc[4 * i + 2] * inv,
                               o_acc[4 * i + 3] * inv);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + obase);
#pragma unroll
        for (int i = 0; i < HD / 8; ++i)
          dst[i] = make_uint4(pack_half2(o_acc[8 * i] * inv, o_acc[8 * i + 1] * inv),
                              pack_half2(o_acc[8 * i + 2] * inv, o_acc[8 * i + 3] * inv),
                              pack_half2(o_acc[8 * i + 4] * inv, o_acc[8 * i + 5] * inv),
                              pack_half2(o_acc[8 * i + 6] * inv, o_acc[8 * i + 7] * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------
// partial-result merge (ring attention combine step)
// ---------------------------------------------------------------------------

__global__ void attn_merge_kernel(float* __restrict__ o_acc, float* __restrict__ lse_acc,
                                  const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                  long long ld, long long bs, __half* __restrict__ out16, long long ld16,
                                  long long bs16, int heads, int seq_q, int hd) {
  // one warp per (b, h, row); lanes stride over head_dim
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(gridDim.y) * heads * seq_q;  // gridDim.y = batch
  (void)rows;
  const int b = blockIdx.y;
  if (gw >= static_cast<long long>(heads) * seq_q) return;
  const int h = static_cast<int>(gw / seq_q);
  const int i = static_cast<int>(gw % seq_q);
  const long long li = (static_cast<long long>(b) * heads + h) * seq_q + i;
  const float la = lse_acc[li], lb = lse_part[li];
  const float L = fmaxf(la, lb) == -INFINITY ? -INFINITY : fmaxf(la, lb) + log1pf(__expf(-fabsf(la - lb)));
  const float wa = la == -INFINITY ? 0.f : __expf(la - L);
  const float wb = lb == -INFINITY ? 0.f : __expf(lb - L);
  const long long base = static_cast<long long>(b) * bs + static_cast<long long>(i) * ld + static_cast<long long>(h) * hd;
  const long long base16 = static_cast<long long>(b) * bs16 + static_cast<long long>(i) * ld16 + static_cast<long long>(h) * hd;
  for (int d = lane; d < hd; d += 32) {
    const float v = o_acc[base + d] * wa + o_part[base + d] * wb;
    o_acc[base + d] = v;
    if (out16 != nullptr) out16[base16 + d] = __float2half_rn(v);
  }
  if (lane == 0) lse_acc[li] = L;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int HD>
static int launch_flash(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const AttnKParams& kp, dim3 grid, cudaStream_t stream) {
  using L = AttnSmem<HD>;
  auto kern = flash_fwd_tcgen05<HD>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(flash): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  kern<<<grid, kAttnThreads, L::kAlloc, stream>>>(tq, tk, tv, kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "flash launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

int flash_fwd(const AttnArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.heads <= 0 || a.seq_q <= 0) return TF_OK;
  if (a.head_dim != 64 && a.head_dim != 128)
    return set_error(TF_ERR_SHAPE, "flash: head_dim=%lld (64 or 128 supported)", a.head_dim);
  if (a.seq_k < 0 || a.seq_q > (1ll << 30) || a.seq_k > (1ll << 30) || a.heads > 65535 || a.batch > 65535)
    return set_error(TF_ERR_SHAPE, "flash: sizes out of range");
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.out))
    return set_error(TF_ERR_ALIGN, "flash: q, k, v and out must be 16-byte aligned");
  if (a.ld_q % 8 || a.ld_kv % 8 || a.bs_q % 8 || a.bs_kv % 8 || a.ld_o % 8 || a.bs_o % 8)
    return set_error(TF_ERR_ALIGN, "flash: pitches must be multiples of 8 elements");
  const long long inner = a.heads * a.head_dim;
  if (a.ld_q < inner || a.ld_kv < inner || a.ld_o < inner)
    return set_error(TF_ERR_SHAPE, "flash: token pitch smaller than heads*head_dim");
  if (a.out == nullptr || a.q == nullptr || a.k == nullptr || a.v == nullptr)
    return set_error(TF_ERR_SHAPE, "flash: null operand");

  const long long seq_k_map = a.seq_k > 0 ? a.seq_k : 1;
  const long long bs_q = a.batch > 1 ? a.bs_q : a.ld_q * a.seq_q;
  const long long bs_kv = a.batch > 1 ? a.bs_kv : a.ld_kv * seq_k_map;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_3d_f16(&tq, a.q, inner, a.seq_q, a.batch, a.ld_q, bs_q > 0 ? bs_q : a.ld_q, 64, kAttnBM);
  if (rc) return rc;
  rc = make_tmap_3d_f16(&tk, a.k, inner, seq_k_map, a.batch, a.ld_kv, bs_kv > 0 ? bs_kv : a.ld_kv, 64, kAttnBN);
  if (rc) return rc;
  rc = make_tmap_3d_f16(&tv, a.v, inner, seq_k_map, a.batch, a.ld_kv, bs_kv > 0 ? bs_kv : a.ld_kv, 64, kAttnBN);
  if (rc) return rc;

  AttnKParams kp;
  kp.out = a.out;
  kp.ld_o = a.ld_o;
  kp.bs_o = a.bs_o;
  kp.lse = a.lse;
  kp.key_valid = a.key_valid;
  kp.heads = static_cast<int>(a.heads);
  kp.seq_q = static_cast<int>(a.seq_q);
  kp.seq_k = static_cast<int>(a.seq_k);
  kp.q_tiles = static_cast<int>((a.seq_q + kAttnBM - 1) / kAttnBM);
  kp.scale_log2 = a.scale * 1.4426950408889634f;
  kp.q_pos0 = a.q_pos0;
  kp.k_pos0 = a.k_pos0;
  kp.flags = a.flags;
  kp.status = device_status_ptr();
  if (kp.status == nullptr) return last_error_code();
  dim3 grid(kp.q_tiles, static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch));
  return a.head_dim == 64 ? launch_flash<64>(tq, tk, tv, kp, grid, stream)
                          : launch_flash<128>(tq, tk, tv, kp, grid, stream);
}

int attn_merge(const MergeArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.heads <= 0 || a.seq_q <= 0) return TF_OK;
  if (a.head_dim <= 0 || a.batch > 65535) return set_error(TF_ERR_SHAPE, "merge: bad sizes");
  if (a.o_acc == nullptr || a.lse_acc == nullptr || a.o_part == nullptr || a.lse_part == nullptr)
    return set_error(TF_ERR_SHAPE, "merge: null operand");
  const long long warps = a.heads * a.seq_q;
  const long long blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffffll) return set_error(TF_ERR_SHAPE, "merge: too many rows");
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(a.batch));
  attn_merge_kernel<<<grid, 256, 0, stream>>>(a.o_acc, a.lse_acc, a.o_part, a.lse_part, a.ld, a.bs,
                                              static_cast<__half*>(a.out16), a.ld16, a.bs16,
                                              static_cast<int>(a.heads), static_cast<int>(a.seq_q),
                                              static_cast<int>(a.head_dim));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "merge launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
