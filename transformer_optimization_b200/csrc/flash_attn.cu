// Flash attention forward on the 5th-generation tensor cores.
//
//   out_i = sum_j softmax_j(scale * q_i . k_j) v_j       (fp16 in, fp32 math)
//
// Replaces the attention of the reference's fp32-model fast path
// (F.scaled_dot_product_attention / _short_attn_kernel / _flash_attn_kernel,
// torch_transformer_benchmark.py:4146-4161, 1193-1418). Like the reference's
// flash kernel it never materialises the score matrix: scores and
// probabilities live in TMEM, one 128-key block at a time, with a running
// max per query row and exp2 with the scale folded into log2(e)
// (torch_transformer_benchmark.py:1427-1428).
//
// One CTA = two 128-query tiles of one (batch, head), 384 threads:
//   warp 0        TMA producer: both Q tiles, then the K_j blocks
//   warp 1        TMEM allocator + single-thread tcgen05.mma issuer
//   warp 2        TMA producer of the V_j blocks
//   warps 4..7    softmax of tile 0 (thread = query row)
//   warps 8..11   softmax of tile 1
// Per key block j and tile t (a "pair" q, issued in the order t0 j0, t1 j0,
// t0 j1, ...) the MMA thread issues
//   S_q = Q_t K_j^T   -> one of NS TMEM slots (fp32, 128 columns)
//   O_t += P_q V_j    -> TMEM (fp32, accumulated over all blocks), with P_q
//                        read from TMEM (tcgen05.mma A-from-TMEM form)
// in the order S_0 .. S_{NS-1}, then PV_q, S_{q+NS} for each q. The softmax
// writes P_q as packed fp16 over the first 64 columns of S_q's slot, so a
// slot is free again once PV_q has been issued (the tensor core executes in
// issue order). The two softmax warpgroups take turns for the exponentials,
// so one tile's exp phase overlaps the other tile's TMEM load and row max.
//
// Online softmax with lazy rescaling: a row keeps a reference max m; P =
// exp2(s*c - m) is computed against it, and O (and l) are rescaled in TMEM
// only when the row max grows by more than 8 (log2 units), so P <= 2^8 stays
// well inside fp16. The final O/l is the exact softmax either way. The row
// sum l adds the fp32 probabilities before their rounding to fp16.
//
// The kernel also emits the natural-log sum-exp per row, used to merge the
// partial results of context-parallel ring attention exactly.
//
// Operand type DT: fp16 (the fp32 model's compute type, and fp16 models) or
// bf16 (bf16 models, whose eager attention rounds the probabilities to bf16
// before P V: torch_transformer_benchmark.py:190-191); P is rounded to DT.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kAttnBM = 128;  // query rows per tile
constexpr int kAttnBN = 128;  // keys per block
constexpr int kAttnTiles = 2;
constexpr int kAttnThreads = 384;
constexpr float kRescaleThreshold = 8.0f;
// Register split: the kernel is built at 168 registers/thread (384 threads,
// 64512 per CTA); warpgroup 0 (producers, MMA) drops to 40 and the two
// softmax warpgroups rise to 232: 128*40 + 256*232 = 64512, the launch pool.
constexpr int kRegsLaunch = 168;
constexpr int kRegsLow = 40;
constexpr int kRegsHigh = 232;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kAttnThreads * kRegsLaunch, "register split exceeds the pool");

struct AttnKParams {
  void* out;
  long long ld_o, bs_o;
  float* lse;
  const uint8_t* key_valid;
  int heads, seq_q, seq_k;
  int q_blocks;      // CTAs along the query axis (256 rows each)
  float scale_log2;  // scale * log2(e); log2(e) with RND (the scores arrive scaled)
  float scale;       // the softmax scale, applied in the score type with RND
  long long q_pos0, k_pos0;
  int flags;
  int* status;
};

template <int HD>
struct AttnCfg {
  // S = Q K^T for successive (tile, key block) pairs goes round a ring of kNS
  // TMEM slots; the softmax overwrites the first 64 columns of its slot with
  // P (fp16 pairs), which the PV product reads straight from TMEM. A slot is
  // reused by S of the pair kNS later, issued after that PV: the tensor core
  // runs the MMAs of this thread in issue order.
  static constexpr int kNS = HD == 64 ? 3 : 2;
  static constexpr int kKStages = HD == 64 ? 4 : 2;
  static constexpr int kVStages = HD == 64 ? 4 : 2;
  static constexpr int kTileBytes = 128 * HD * 2;  // a 128-row x HD fp16 tile
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kAttnTiles * kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kVStages * kTileBytes;
  // q_full, k_full/empty[KS], v_full/empty[VS], s_full[NS],
  // p_full[2 tiles x 2 alternating], o_full[2], turn[2], drain[2], pv_done[NS]
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + kNS + 4 + 2 + 2 + 2 + kNS;
  static constexpr int kBytes = kBarOff + kNumBars * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
  // TMEM columns: S/P slots at 0, 128, ..; O_t at kNS*128 + t*HD (512 in all)
  static constexpr uint32_t kTmS = 0;
  static constexpr uint32_t kTmO = kNS * 128;
  static_assert(kNS * 128 + kAttnTiles * HD <= 512, "TMEM budget");
};

// volatile: the exp-unit sweep must stay between the turn wait and arrive
__device__ __forceinline__ float ex2_f32(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t ex2_f16x2(uint32_t h) {
  uint32_t r;
  asm volatile("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(h));
  return r;
}

// 2^t as a binary16 bit pattern, computed on the FMA/integer pipes (not the
// exp unit), for t <= 8 (t may be -inf). Cody-Waite style reduction t = n + f
// with n = round-to-nearest(t - 1/2), f in [0, 1]; 2^f from a degree-3
// minimax polynomial with p(0) = 1 (coefficients fitted for this library by a
// Remez iteration; max relative error 8.6e-5, below half an fp16 ulp); then
// the binary16 pattern (n + 15) * 1024 + round(1024 * 2^f) - 1024, where a
// mantissa that rounds up to 2048 carries into the exponent field. Results
// below 2^-14 (fp16 subnormals) flush to zero.
// 2^t in fp32 on the FMA/integer pipes (not the exp unit), for t <= 8 (t
// may be -inf): the same reduction and degree-3 polynomial as
// exp2_f16_bits_fma (relative error <= 8.6e-5, below half an fp16 ulp, which
// is the precision P is used at), then n added to the exponent field.
// Results below 2^-126 are 0.
__device__ __forceinline__ float exp2_f32_fma(float t) {
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const float y = (t - 0.5f) + kRound;
  const float f = t - (y - kRound);  // in [0, 1]
  float p = fmaf(f, 0.07706703990697861f, 0.22764499485492706f);
  p = fmaf(p, f, 0.6951167583465576f);
  p = fmaf(p, f, 1.0f);
  // the low 9 bits of bits(y) hold n mod 512 (kRound's are zero), so
  // bits(y) << 23 is n << 23 mod 2^32
  const float r = __uint_as_float(__float_as_uint(p) + (__float_as_uint(y) << 23));
  return t < -126.0f ? 0.f : r;
}

__device__ __forceinline__ uint32_t exp2_f16_bits_fma(float t) {
  const float kRound = 12582912.0f;  // 1.5 * 2^23: y = x + kRound keeps round(x) in the low bits of y
  const float y = (t - 0.5f) + kRound;
  const float f = t - (y - kRound);
  float p = fmaf(f, 0.07706703990697861f, 0.22764499485492706f);
  p = fmaf(p, f, 0.6951167583465576f);
  p = fmaf(p, f, 1.0f);
  const float q = fmaf(p, 1024.0f, kRound);  // low bits: round(1024 * p)
  // (bits(y) - B) * 1024 + (bits(q) - B) + 14336, B = bits(kRound), mod 2^32
  const uint32_t h = __float_as_uint(y) * 1024u + __float_as_uint(q) + (14336u - 0x4B400000u * 1025u);
  return t < -14.0f ? 0u : (h & 0xFFFFu);
}

__device__ __forceinline__ uint32_t pack_f16x2_rn(float a, float b) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  return h;
}

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float a, float b) {
  uint32_t h;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  return h;
}

// a probability pair in the PV operand type (a in the low half)
template <int DT>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  if constexpr (DT == kDtBF16) {
    return pack_bf16x2_rn(a, b);
  } else {
    return pack_f16x2_rn(a, b);
  }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Scale columns [0, NO) of this thread's O row in TMEM by alpha.
template <int NO>
__device__ __forceinline__ void rescale_o(uint32_t taddr, float alpha) {
#pragma unroll
  for (int c = 0; c < NO / 32; ++c) {
    uint32_t v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
    tmem_st32(taddr + c * 32, v);
  }
  if constexpr (NO % 32 == 16) {
    uint32_t v[16];
    tmem_ld16(taddr + (NO / 32) * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
    tmem_st16(taddr + (NO / 32) * 32, v);
  }
  tmem_wait_st();
}

// RND (TF_ATTN_ROUND_SCORES, half-precision models): the scores are those of
// the eager model run in the operand type T, T(T(q . k) * scale)
// (torch_transformer_benchmark.py:173: matmul in T, then the scale in T),
// before the fp32 softmax (:188); without it the scores stay fp32.
template <int HD, bool EXP16, int POLY, int DT, bool RND = false>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_fwd_tcgen05(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, AttnKParams p) {
  using C = AttnCfg<HD>;
  constexpr int KS = C::kKStages;
  constexpr int VS = C::kVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  constexpr int NS = C::kNS;
  uint64_t* s_full = v_empty + VS;
  uint64_t* p_full = s_full + NS;  // [tile * 2 + (block & 1)]: alternating, so no waiter falls two phases behind
  uint64_t* o_full = p_full + 4;   // [tile]: every PV of the tile so far has landed in O
  uint64_t* turn = o_full + 2;     // exp-phase hand-off between the two softmax warpgroups
  uint64_t* drain = turn + 2;       // [issuer]: end-of-kernel drain of each MMA issuer
  uint64_t* pv_done = drain + 2;    // [slot]: the PV that read this slot's P has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + NS);

  const int warp = warp_id();
  const int lane = lane_id();
  const int qb = p.q_blocks - 1 - static_cast<int>(blockIdx.x);  // longest (causal) first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = qb * (kAttnBM * kAttnTiles);
  const bool causal = (p.flags & TF_ATTN_CAUSAL) != 0;

  // key blocks needed by each tile
  int nblk[kAttnTiles];
#pragma unroll
  for (int t = 0; t < kAttnTiles; ++t) {
    const int tq0 = q0 + t * kAttnBM;
    long long k_end = tq0 < p.seq_q ? p.seq_k : 0;
    if (causal && k_end > 0) {
      const long long last_q = p.q_pos0 + tq0 + kAttnBM - 1;
      const long long lim = last_q - p.k_pos0 + 1;
      if (lim < k_end) k_end = lim;
    }
    nblk[t] = k_end <= 0 ? 0 : static_cast<int>((k_end + kAttnBN - 1) / kAttnBN);
  }
  const int nmax = nblk[0] > nblk[1] ? nblk[0] : nblk[1];
  // (tile, key block) pairs in issue order: (0, j), (1, j) while both tiles
  // need block j, then the longer tile alone
  const int nmin = nblk[0] < nblk[1] ? nblk[0] : nblk[1];
  const int t_long = nblk[0] > nblk[1] ? 0 : 1;
  const int n_pairs = nblk[0] + nblk[1];

  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmQ);
    tma_prefetch_map(&tmK);
    tma_prefetch_map(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < NS; ++i) mbar_init(&s_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&o_full[i], 1);
      mbar_init(&turn[i], 128);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    for (int i = 0; i < NS; ++i) mbar_init(&pv_done[i], 1);
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
  // everything above touched only this CTA's shared memory and TMEM
  pdl_wait();
  pdl_trigger();
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
  if (warp == 0) {
    if (lane == 0 && nmax > 0) {
      // ---------------- Q + K producer ----------------
      mbar_arrive_expect_tx(q_full, kAttnTiles * C::kTileBytes);
#pragma unroll
      for (int t = 0; t < kAttnTiles; ++t)
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_3d(smem + C::kQOff + t * C::kTileBytes + c * 16384, &tmQ, q_full, h * HD + c * 64,
                      q0 + t * kAttnBM, b);
      int j = 0;
      for (; j < nmax; ++j) {
        const int s = j % KS;
        if (!mbar_wait(&k_empty[s], ((j / KS) & 1) ^ 1, p.status, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(&k_full[s], C::kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_3d(smem + C::kKOff + s * C::kTileBytes + c * 16384, &tmK, &k_full[s], h * HD + c * 64,
                      j * kAttnBN, b);
      }
      mbar_wait(q_full, 0, p.status, kDevTimeoutDrain);
      for (int i = (j > KS ? j - KS : 0); i < j; ++i)
        mbar_wait(&k_full[i % KS], (i / KS) & 1, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 2) {
    if (lane == 0 && nmax > 0) {
      // ---------------- V producer ----------------
      int j = 0;
      for (; j < nmax; ++j) {
        const int s = j % VS;
        if (!mbar_wait(&v_empty[s], ((j / VS) & 1) ^ 1, p.status, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(&v_full[s], C::kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_3d(smem + C::kVOff + s * C::kTileBytes + c * 16384, &tmV, &v_full[s], h * HD + c * 64,
                      j * kAttnBN, b);
      }
      for (int i = (j > VS ? j - VS : 0); i < j; ++i)
        mbar_wait(&v_full[i % VS], (i / VS) & 1, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1 || warp == 3) {
    if (lane == 0 && nmax > 0) {
      // ---------------- MMA issuers ----------------
      // Two threads feed the tensor core: warp 1 issues the S = Q K^T
      // products, warp 3 the O += P V products. Each stream waits only on
      // its own inputs, so neither stalls behind the other's barrier waits
      // and commits (the tensor core queue is shallow). A slot's next S
      // waits for the completion of the PV that read the slot's P (pv_done).
      constexpr uint32_t idesc_s = idesc_16_f32(DT, kAttnBM, kAttnBN);     // K-major Q, K-major K
      constexpr uint32_t idesc_o = idesc_16_f32(DT, kAttnBM, HD, false, true);  // K-major P, MN-major V
      const uint32_t sbase = smem_u32(smem);
      auto pair_of = [&](int q, int& t, int& j) {
        if (q < 2 * nmin) {
          j = q >> 1;
          t = q & 1;
        } else {
          j = nmin + (q - 2 * nmin);
          t = t_long;
        }
      };
      // the last pair (in issue order) that reads key block j
      auto last_user = [&](int t, int j) { return t == 1 || j >= nblk[1]; };
      bool ok = true;
      if (warp == 1) {
        ok = mbar_wait(q_full, 0, p.status, kDevTimeoutMma);
        for (int q = 0; q < n_pairs && ok; ++q) {
          int t, j;
          pair_of(q, t, j);
          const int slot = q % NS;
          if (q >= NS && !(ok = mbar_wait(&pv_done[slot], ((q - NS) / NS) & 1, p.status, kDevTimeoutMma))) break;
          if (!(ok = mbar_wait(&k_full[j % KS], (j / KS) & 1, p.status, kDevTimeoutMma))) break;
          tc_fence_after();
          const uint32_t qa = sbase + C::kQOff + t * C::kTileBytes;
          const uint32_t ka = sbase + C::kKOff + (j % KS) * C::kTileBytes;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
            umma_f16_ss(tmem_base + C::kTmS + slot * 128, smem_desc_sw128(qa + off, 16, 1024),
                        smem_desc_sw128(ka + off, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[slot]);
          if (last_user(t, j)) umma_commit(&k_empty[j % KS]);
        }
      } else {
        for (int q = 0; q < n_pairs && ok; ++q) {
          int t, j;
          pair_of(q, t, j);
          const int slot = q % NS;
          if (!(ok = mbar_wait(&v_full[j % VS], (j / VS) & 1, p.status, kDevTimeoutMma))) break;
          if (!(ok = mbar_wait(&p_full[t * 2 + (j & 1)], (j >> 1) & 1, p.status, kDevTimeoutMma))) break;
          tc_fence_after();
          const uint32_t va = sbase + C::kVOff + (j % VS) * C::kTileBytes;
          // P: 128 keys = 64 TMEM columns, 8 per MMA; V: MN-major, 8-key
          // groups at 1024 B (SBO), 64-wide head-dim blocks at 16 KB (LBO)
#pragma unroll
          for (int k = 0; k < kAttnBN / 16; ++k)
            umma_f16_ts(tmem_base + C::kTmO + t * HD, tmem_base + C::kTmS + slot * 128 + k * 8,
                        smem_desc_sw128(va + k * 2048, 16384, 1024), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(&pv_done[slot]);
          umma_commit(&o_full[t]);
          if (last_user(t, j)) umma_commit(&v_empty[j % VS]);
        }
      }
      // drain: every MMA this thread issued completes before TMEM is released
      uint64_t* d = &drain[warp == 1 ? 0 : 1];
      umma_commit(d);
      mbar_wait(d, 0, p.status, kDevTimeoutDrain);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ---------------- softmax (warps 4..11) ----------------
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile
    const int row = q0 + t * kAttnBM + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tm_s = tmem_base + lane_off + C::kTmS;
    const uint32_t tm_o = tmem_base + lane_off + C::kTmO + t * HD;
    const long long q_glob = p.q_pos0 + row;
    const uint8_t* kvalid = p.key_valid ? p.key_valid + static_cast<long long>(b) * p.seq_k : nullptr;
    const int nb = nblk[t];
    const int n_pp = nmin;  // blocks where both tiles take turns
    const float c = p.scale_log2;

    float m_ref = -INFINITY;  // reference max (scaled log2 domain)
    float l = 0.f;            // row sum
    bool ok = true;

    for (int j = 0; j < nb; ++j) {
      const int q = j < nmin ? 2 * j + t : 2 * nmin + (j - nmin);  // issue order of (t, j)
      const int slot = q % NS;
      if (!(ok = mbar_wait(&s_full[slot], (q / NS) & 1, p.status, kDevTimeoutSoftmax))) break;
      tc_fence_after();
      float s[128];
      {
        uint32_t v[128];
        tmem_ld128(tm_s + slot * 128, v);  // the whole S row in one load, one wait
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(v[i]);
      }
      if constexpr (RND) {
#pragma unroll
        for (int i = 0; i < 128; i += 2) {
          const float2 qk = unpack2<DT>(pack2<DT>(s[i], s[i + 1]));                   // T(q . k)
          const float2 sc = unpack2<DT>(pack2<DT>(qk.x * p.scale, qk.y * p.scale));  // T(T(q . k) * scale)
          s[i] = sc.x;
          s[i + 1] = sc.y;
        }
      }

      // ---- masking (tails, causal diagonal, key padding) ----
      const long long kbase = static_cast<long long>(j) * kAttnBN;
      long long lim_ll = p.seq_k - kbase;
      if (causal) {
        const long long cl = q_glob - p.k_pos0 - kbase + 1;
        lim_ll = cl < lim_ll ? cl : lim_ll;
      }
      const int lim = lim_ll < 0 ? 0 : (lim_ll > kAttnBN ? kAttnBN : static_cast<int>(lim_ll));
      if (__any_sync(0xffffffffu, lim < kAttnBN)) {
#pragma unroll
        for (int i = 0; i < 128; ++i) s[i] = i < lim ? s[i] : -INFINITY;
      }
      if (kvalid != nullptr) {
        const uint8_t* kv = kvalid + kbase;
        const long long rem = p.seq_k - kbase;
        const int avail = rem >= kAttnBN ? kAttnBN : static_cast<int>(rem);
        const bool fast = avail == kAttnBN && (reinterpret_cast<uintptr_t>(kv) & 15) == 0;
#pragma unroll
        for (int g = 0; g < 128; g += 16) {
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (fast) {
            const uint4 q4 = __ldg(reinterpret_cast<const uint4*>(kv + g));
            w[0] = q4.x;
            w[1] = q4.y;
            w[2] = q4.z;
            w[3] = q4.w;
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (g + i < avail) w[i >> 2] |= static_cast<uint32_t>(kv[g + i]) << (8 * (i & 3));
          }
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (((w[i >> 2] >> (8 * (i & 3))) & 0xffu) == 0u) s[g + i] = -INFINITY;
        }
      }

      // ---- row max: eight 3-input-max chains, then a short tree ----
      // chain k covers s[k + 8*i] for i = 0..15 (all 128 columns)
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmax3f(s[k], s[8 + k], s[16 + k]);
#pragma unroll
      for (int base = 24; base < 120; base += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmax3f(mx[k], s[base + k], s[base + 8 + k]);
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], s[120 + k]);
      mx[0] = fmax3f(mx[0], mx[1], mx[2]);
      mx[3] = fmax3f(mx[3], mx[4], mx[5]);
      mx[0] = fmax3f(mx[0], mx[3], fmaxf(mx[6], mx[7]));
      const float m_row = mx[0] * c;

      // ---- lazy rescale of O (and l) ----
      const bool need = m_row > m_ref + kRescaleThreshold;
      if (j == 0) {
        m_ref = m_row;
      } else if (__any_sync(0xffffffffu, need)) {
        const float m_new = fmaxf(m_ref, m_row);
        const float alpha = m_ref == -INFINITY ? 0.f : ex2_f32(m_ref - m_new);
        // every PV so far (the last is block j-1) must have landed in O
        if (!(ok = mbar_wait(&o_full[t], (j - 1) & 1, p.status, kDevTimeoutSoftmax))) break;
        tc_fence_after();
        rescale_o<HD>(tm_o, alpha);
        l *= alpha;
        m_ref = m_new;
      }
      const float m_use = m_ref == -INFINITY ? 0.f : m_ref;

      // ---- exponentials ----
      // Only the exp-unit instructions run in turns with the other tile's
      // warpgroup (tile 0 of block j after tile 1 of block j-1, tile 1 of
      // block j after tile 0 of block j): the scale/shift and packing before
      // the turn, the FMA-pipe exponentials, the row sum and the P store
      // after it, where they overlap the other group's exp-unit sweep.
      uint32_t pk[64];
      float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 128; ++i) s[i] = fmaf(s[i], c, -m_use);
      if constexpr (EXP16) {
#pragma unroll
        for (int i = POLY; i < 64; ++i) pk[i] = pack_f16x2_rn(s[2 * i], s[2 * i + 1]);
      }
      if (j < n_pp && (t == 1 || j > 0)) {
        const uint32_t par = t == 0 ? ((j - 1) & 1) : (j & 1);
        if (!(ok = mbar_wait(&turn[t], par, p.status, kDevTimeoutSoftmax))) break;
      }
      if constexpr (EXP16) {
        // POLY of the 64 pairs on the FMA pipes, the rest on the exp unit
#pragma unroll
        for (int i = POLY; i < 64; ++i) pk[i] = ex2_f16x2(pk[i]);
      } else {
        // 2*POLY of the 128 on the FMA pipes, the rest on the exp unit
#pragma unroll
        for (int i = 2 * POLY; i < 128; ++i) s[i] = ex2_f32(s[i]);
      }
      if (j < n_pp) mbar_arrive(&turn[1 - t]);
      if constexpr (EXP16) {
#pragma unroll
        for (int i = 0; i < POLY; ++i)
          pk[i] = exp2_f16_bits_fma(s[2 * i]) | (exp2_f16_bits_fma(s[2 * i + 1]) << 16);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pk[i]));
          ls[i & 7] += f.x + f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 2 * POLY; ++i) s[i] = exp2_f32_fma(s[i]);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          pk[i] = pack_p<DT>(s[2 * i], s[2 * i + 1]);
          ls[i & 7] += s[2 * i] + s[2 * i + 1];
        }
      }
      l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));

      // P into the first 64 columns of this pair's S slot (already read)
      tmem_st64(tm_s + slot * 128, pk);
      tmem_wait_st_all();
      tc_fence_before();
      mbar_arrive(&p_full[t * 2 + (j & 1)]);
    }

    // ---------------- epilogue ----------------
    if (ok) {
      float inv = 0.f;
      uint32_t ov[HD];
      if (nb > 0) {
        if (!(ok = mbar_wait(&o_full[t], (nb - 1) & 1, p.status, kDevTimeoutSoftmax))) {
          // fall through to the barrier; nothing is written
        } else {
          tc_fence_after();
          if constexpr (HD == 128) {
            tmem_ld128(tm_o, ov);
          } else {
            tmem_ld64(tm_o, ov);
          }
          tmem_wait_ld();
        }
      } else {
#pragma unroll
        for (int i = 0; i < HD; ++i) ov[i] = 0u;
      }
      if (ok && row < p.seq_q) {
        inv = l > 0.f ? 1.f / l : 0.f;
        if (p.lse != nullptr)
          p.lse[(static_cast<long long>(b) * p.heads + h) * p.seq_q + row] =
              l > 0.f ? (m_ref + __log2f(l)) * 0.69314718055994531f : -INFINITY;
        const long long obase =
            static_cast<long long>(b) * p.bs_o + static_cast<long long>(row) * p.ld_o + h * HD;
        if (p.flags & TF_ATTN_OUT_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase);
#pragma unroll
          for (int i = 0; i < HD / 4; ++i)
            dst[i] = make_float4(__uint_as_float(ov[4 * i]) * inv, __uint_as_float(ov[4 * i + 1]) * inv,
                                 __uint_as_float(ov[4 * i + 2]) * inv, __uint_as_float(ov[4 * i + 3]) * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + obase);
#pragma unroll
          for (int i = 0; i < HD / 8; ++i)
            dst[i] = make_uint4(
                pack2<DT>(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv),
                pack2<DT>(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv),
                pack2<DT>(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv),
                pack2<DT>(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv));
        }
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
  pdl_wait();
  pdl_trigger();
  // one warp per (b, h, row); lanes stride over head_dim
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  if (gw >= static_cast<long long>(heads) * seq_q) return;
  const int h = static_cast<int>(gw / seq_q);
  const int i = static_cast<int>(gw % seq_q);
  const long long li = (static_cast<long long>(b) * heads + h) * seq_q + i;
  const float la = lse_acc[li], lb = lse_part[li];
  const float mx = fmaxf(la, lb);
  const float L = mx == -INFINITY ? -INFINITY : mx + log1pf(__expf(-fabsf(la - lb)));
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

// The same merge with one warp per (batch, token row) covering all heads:
// lanes 0..heads-1 compute their head's weights once, and the row's
// heads*hd values move as float4 with their head's weights taken from that
// lane (heads <= 32, hd % 4 == 0, 16-byte aligned rows). Per element the
// arithmetic is the one above.
__global__ void attn_merge_rows_kernel(float* __restrict__ o_acc, float* __restrict__ lse_acc,
                                       const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                       long long ld, long long bs, __half* __restrict__ out16, long long ld16,
                                       long long bs16, int heads, int seq_q, int hd, long long rows) {
  pdl_wait();
  pdl_trigger();
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows) return;  // whole warps leave together
  const int b = static_cast<int>(gw / seq_q);
  const int i = static_cast<int>(gw % seq_q);
  float wa = 0.f, wb = 0.f;
  if (lane < heads) {
    const long long li = (static_cast<long long>(b) * heads + lane) * seq_q + i;
    const float la = lse_acc[li], lb = lse_part[li];
    const float mx = fmaxf(la, lb);
    const float L = mx == -INFINITY ? -INFINITY : mx + log1pf(__expf(-fabsf(la - lb)));
    wa = la == -INFINITY ? 0.f : __expf(la - L);
    wb = lb == -INFINITY ? 0.f : __expf(lb - L);
    lse_acc[li] = L;
  }
  float4* pa = reinterpret_cast<float4*>(o_acc + static_cast<long long>(b) * bs + static_cast<long long>(i) * ld);
  const float4* pb =
      reinterpret_cast<const float4*>(o_part + static_cast<long long>(b) * bs + static_cast<long long>(i) * ld);
  uint2* p16 = out16 == nullptr ? nullptr
                                : reinterpret_cast<uint2*>(out16 + static_cast<long long>(b) * bs16 +
                                                           static_cast<long long>(i) * ld16);
  const int nv = heads * hd / 4;
  for (int base = 0; base < nv; base += 32) {
    const int q = base + lane;
    const int h = q < nv ? (4 * q) / hd : 0;
    const float ca = __shfl_sync(0xffffffffu, wa, h);
    const float cb = __shfl_sync(0xffffffffu, wb, h);
    if (q < nv) {
      const float4 x = pa[q], y = __ldcs(pb + q);
      const float4 v = make_float4(x.x * ca + y.x * cb, x.y * ca + y.y * cb, x.z * ca + y.z * cb, x.w * ca + y.w * cb);
      pa[q] = v;
      if (p16 != nullptr) {
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        __stcs(p16 + q, make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1)));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int HD, bool EXP16, int POLY, int DT = kDtF16, bool RND = false>
static int launch_flash(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const AttnKParams& kp, dim3 grid, cudaStream_t stream) {
  using C = AttnCfg<HD>;
  auto kern = flash_fwd_tcgen05<HD, EXP16, POLY, DT, RND>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    // The in-kernel register split assumes the launch pool of exactly
    // kRegsLaunch registers per thread; refuse anything else rather than
    // risk a split that can never be satisfied.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncGetAttributes(flash): %s", cudaGetErrorString(e));
    if (fa.numRegs != kRegsLaunch)
      return set_error(TF_ERR_LAUNCH, "flash kernel built with %d registers/thread, expected %d", fa.numRegs,
                       kRegsLaunch);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(flash): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  cudaError_t e = launch_k(kern, grid, dim3(kAttnThreads), C::kAlloc, stream, tq, tk, tv, kp);
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
  kp.q_blocks = static_cast<int>((a.seq_q + kAttnBM * kAttnTiles - 1) / (kAttnBM * kAttnTiles));
  const bool rnd = (a.flags & TF_ATTN_ROUND_SCORES) != 0;
  kp.scale = a.scale;
  kp.scale_log2 = rnd ? 1.4426950408889634f : a.scale * 1.4426950408889634f;
  kp.q_pos0 = a.q_pos0;
  kp.k_pos0 = a.k_pos0;
  kp.flags = a.flags;
  kp.status = device_status_ptr();
  if (kp.status == nullptr) return last_error_code();
  dim3 grid(kp.q_blocks, static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch));
  const bool exp16 = (a.flags & TF_ATTN_EXP_F16X2) != 0;
  // probability pairs per row and key block whose exponentials run on the
  // FMA pipes instead of the exp unit (flags bits 8..15)
  const int poly = (a.flags >> 8) & 0xFF;
  if (poly != 0 && poly != 8 && poly != 16 && poly != 24)
    return set_error(TF_ERR_SHAPE, "flash: FMA-pipe exp pairs must be 0, 8, 16 or 24");
  if (exp16 && poly != 0 && poly != 16)
    return set_error(TF_ERR_SHAPE, "flash: with TF_ATTN_EXP_F16X2 the FMA-pipe exp pairs must be 0 or 16");
  if (rnd && (exp16 || poly != 0))
    return set_error(TF_ERR_SHAPE, "flash: TF_ATTN_ROUND_SCORES takes neither TF_ATTN_EXP_F16X2 nor FMA-pipe exponentials");
  if (a.flags & TF_ATTN_BF16) {
    // bf16 operands: fp32 exp2 on the exp unit only (the other exponential
    // forms produce fp16 bits)
    if (exp16 || poly != 0)
      return set_error(TF_ERR_SHAPE, "flash: TF_ATTN_BF16 takes neither TF_ATTN_EXP_F16X2 nor FMA-pipe exponentials");
    if (rnd)
      return a.head_dim == 64 ? launch_flash<64, false, 0, kDtBF16, true>(tq, tk, tv, kp, grid, stream)
                              : launch_flash<128, false, 0, kDtBF16, true>(tq, tk, tv, kp, grid, stream);
    return a.head_dim == 64 ? launch_flash<64, false, 0, kDtBF16>(tq, tk, tv, kp, grid, stream)
                            : launch_flash<128, false, 0, kDtBF16>(tq, tk, tv, kp, grid, stream);
  }
  if (rnd)
    return a.head_dim == 64 ? launch_flash<64, false, 0, kDtF16, true>(tq, tk, tv, kp, grid, stream)
                            : launch_flash<128, false, 0, kDtF16, true>(tq, tk, tv, kp, grid, stream);
#define TFB_FLASH(E, P)                                                            \
  return a.head_dim == 64 ? launch_flash<64, E, P>(tq, tk, tv, kp, grid, stream) \
                          : launch_flash<128, E, P>(tq, tk, tv, kp, grid, stream);
  if (exp16) {
    if (poly == 16) TFB_FLASH(true, 16)
    TFB_FLASH(true, 0)
  }
  switch (poly) {
    case 8: TFB_FLASH(false, 8)
    case 16: TFB_FLASH(false, 16)
    case 24: TFB_FLASH(false, 24)
    default: TFB_FLASH(false, 0)
  }
#undef TFB_FLASH
}

int attn_merge(const MergeArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.heads <= 0 || a.seq_q <= 0) return TF_OK;
  if (a.head_dim <= 0 || a.batch > 65535) return set_error(TF_ERR_SHAPE, "merge: bad sizes");
  if (a.o_acc == nullptr || a.lse_acc == nullptr || a.o_part == nullptr || a.lse_part == nullptr)
    return set_error(TF_ERR_SHAPE, "merge: null operand");
  const bool rows_form = a.heads <= 32 && a.head_dim % 4 == 0 && a.ld % 4 == 0 && a.bs % 4 == 0 &&
                         aligned16(a.o_acc) && aligned16(a.o_part) &&
                         (a.out16 == nullptr ||
                          (reinterpret_cast<uintptr_t>(a.out16) % 8 == 0 && a.ld16 % 4 == 0 && a.bs16 % 4 == 0));
  if (rows_form) {
    const long long rows = a.batch * a.seq_q;
    const long long blocks = (rows * 32 + 255) / 256;
    if (blocks > 0x7fffffffll) return set_error(TF_ERR_SHAPE, "merge: too many rows");
    launch_k(attn_merge_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, a.o_acc, a.lse_acc,
             a.o_part, a.lse_part, a.ld, a.bs, static_cast<__half*>(a.out16), a.ld16, a.bs16,
             static_cast<int>(a.heads), static_cast<int>(a.seq_q), static_cast<int>(a.head_dim), rows);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "merge launch: %s", cudaGetErrorString(e));
    return TF_OK;
  }
  const long long warps = a.heads * a.seq_q;
  const long long blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffffll) return set_error(TF_ERR_SHAPE, "merge: too many rows");
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(a.batch));
  launch_k(attn_merge_kernel, grid, dim3(256), 0, stream, a.o_acc, a.lse_acc, a.o_part, a.lse_part, a.ld, a.bs,
           static_cast<__half*>(a.out16), a.ld16, a.bs16, static_cast<int>(a.heads), static_cast<int>(a.seq_q),
           static_cast<int>(a.head_dim));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "merge launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
