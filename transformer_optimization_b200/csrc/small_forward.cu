// The whole forward pass of a few-row fp32 model in ONE persistent launch.
//
// For inputs of a few hundred tokens (BASELINE's c1: 256 rows, c2: 64 rows)
// every projection, attention and LayerNorm is microseconds of work, and a
// forward made of ~7 dependent launches per layer is bound by launch and
// dependency latency, not by the tensor cores or HBM. This kernel runs the
// reference's per-layer schedule (torch_transformer_benchmark.py:4003-4326,
// fp32-model fp16-GEMM branch 4130-4199) as a sequence of phases inside one
// cooperative launch of one CTA per SM, with a grid-wide barrier between
// dependent phases:
//
//   LN1(x) -> normed                                  (rows)
//   per layer:
//     QKV  = normed . Wqkv^T + b                      (GEMM tiles, fp16 out)
//     ctx  = softmax(scale . Q K^T [causal]) V        (one CTA per batch x head)
//     part = ctx . Wo^T                               (split-K GEMM, fp32 partials)
//     xr   = x + sum(part) + bo; normed = LN2(xr)     (rows)
//     hid  = gelu(normed . W1^T + b1)                 (GEMM tiles, fp16 out)
//     part = hid . W2^T                               (split-K GEMM)
//     xr  += sum(part) + b2; normed = LN1'(xr)        (rows; after the last
//                                                      layer the final LayerNorm, fp32 out)
//
// The arithmetic is that of the multi-kernel path: fp16 operands with fp32
// accumulation on tcgen05 (TMA-fed 128-row x 32-column tiles, accumulator in
// TMEM), the split-K partials summed in fixed split order, erf GELU on the
// fp32 accumulator, fp32 residual stream and two-pass LayerNorm statistics,
// attention probabilities rounded to fp16 for the P.V product.
//
// CTA roles (256 threads): warp 0 lane 0 issues the TMA loads, warp 1 lane 0
// the MMAs, warps 4..7 (one TMEM lane quarter each) run the GEMM epilogues and
// the attention softmax; all eight warps run the row phases (one warp per
// row). Every wait is bounded (%globaltimer); a wait or barrier that runs out
// records a code in the device status word, the CTA stops issuing work,
// keeps arriving at the grid barriers and drains what it issued.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kSfThreads = 256;
constexpr int kSfBM = 128;
constexpr int kSfBN = 32;
constexpr int kSfBK = 64;
constexpr int kSfStages = 8;
constexpr int kSfMaxLayers = 16;
constexpr int kSfMaxSplits = 32;
constexpr int kSfABytes = kSfBM * kSfBK * 2;          // 16 KB
constexpr int kSfWBytes = kSfBN * kSfBK * 2;          // 4 KB
constexpr int kSfStageBytes = kSfABytes + kSfWBytes;  // 20 KB, a multiple of 1024
constexpr int kSfTileBytes = 128 * 64 * 2;            // an attention Q / K / V tile
constexpr int kSfBarOff = kSfStages * kSfStageBytes;
// full[S], empty[S], acc, attn_in, s_full, p_full, o_full, drain
constexpr int kSfNumBars = 2 * kSfStages + 6;
constexpr int kSfSmemBytes = kSfBarOff + kSfNumBars * 8 + 16;
constexpr int kSfSmemAlloc = kSfSmemBytes + 1024;
constexpr uint32_t kSfTmemCols = 256;  // GEMM accumulator [0, 32); attention S/P [0, 128), O [128, 192)
constexpr uint32_t kSfTmemO = 128;
constexpr int kDevTimeoutBarrier = 107;

static_assert(kSfStages * kSfStageBytes >= 3 * kSfTileBytes, "attention tiles reuse the GEMM stages");

struct SfLayer {
  const float* bqkv;
  const float* bo;
  const float* b1;
  const float* b2;
  const float* n1w;
  const float* n1b;
  const float* n2w;
  const float* n2b;
  float eps1, eps2;
};

struct SfParams {
  CUtensorMap w[kSfMaxLayers][4];  // Wqkv [3D, D], Wo [D, D], W1 [F, D], W2 [D, F]
  CUtensorMap a_normed, a_ctx, a_hidden, a_qkv;
  SfLayer layer[kSfMaxLayers];
  const float* x;  // [M, D] input (never written)
  float* out;      // [M, D] output
  float* xr;       // [M, D] residual stream
  uint16_t* normed;
  uint16_t* qkv;
  uint16_t* ctx;
  uint16_t* hidden;
  float* ws;       // split-K partials [splits][M][D]
  unsigned* bar;   // [0] arrivals, [1] generation (zero before the launch)
  int* status;
  const float* fw;
  const float* fb;
  float feps;
  float scale_log2;  // head_dim^-0.5 * log2(e)
  int B, S, D, H, F, L, M, causal;
  int sp_o, sp_2;  // split counts of the out-projection and FFN-out GEMMs
};

enum SfEpi { kSfEpiBias = 0, kSfEpiGelu = 1, kSfEpiPartial = 2 };

// Counters every thread of the CTA keeps identically, so each barrier's
// phase parity is known to all roles across units and phases.
struct SfState {
  int it;    // TMA ring slots used
  int acc;   // GEMM accumulator completions
  int attn;  // attention units
  bool ok;   // no wait of this CTA has run out
  // producer thread only: one past the ring slot of the last load it issued,
  // and one past the attention unit whose tiles it last loaded (for the drain)
  int it_issued;
  int attn_issued;
};

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* ptr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

// Grid-wide barrier (every CTA is resident: cooperative launch). The
// generation is read before arriving; the last CTA to arrive resets the
// arrival count and advances the generation. Generic stores of the phase are
// released by the arrival and acquired by the spin, and ordered before the
// async proxy (the next phase's TMA reads) on both sides. Returns false when
// the wait ran out or another CTA raised an error.
__device__ bool sf_grid_barrier(unsigned* bar, int* status, bool ok, int* s_flag) {
  fence_proxy_async_global();
  __syncthreads();
  if (threadIdx.x == 0) {
    int good = ok ? 1 : 0;
    const unsigned gen = ld_acquire_u32(&bar[1]);
    __threadfence();
    const unsigned prev = atomicAdd(&bar[0], 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(&bar[0], 0u);
      __threadfence();
      atomicAdd(&bar[1], 1u);
    } else {
      long long next_check = clock64() + kSlowCheckCycles;
      uint64_t t0 = 0;
      while (ld_acquire_u32(&bar[1]) == gen) {
        const long long now = clock64();
        if (now >= next_check) {
          next_check = now + kSlowCheckCycles;
          if (error_raised(status)) {
            good = 0;
            break;
          }
          const uint64_t g = globaltimer_ns();
          if (t0 == 0) {
            t0 = g;
          } else if (g - t0 > kWaitLimitNs) {
            record_error(status, kDevTimeoutBarrier);
            good = 0;
            break;
          }
        }
      }
    }
    __threadfence();
    fence_proxy_async_global();
    if (error_raised(status)) good = 0;
    *s_flag = good;
  }
  __syncthreads();
  return *s_flag != 0;
}

// ---------------------------------------------------------------------------
// GEMM phase: out[M, N] (op) A[M, K] . W[N, K]^T over 128 x 32 tiles, K split
// into `splits` ranges (splits > 1 only with kSfEpiPartial)
// ---------------------------------------------------------------------------
struct SfGemm {
  const CUtensorMap* ma;
  const CUtensorMap* mw;
  int M, N, K, splits, epi;
  const float* bias;
  uint16_t* out16;  // kSfEpiBias / kSfEpiGelu, row pitch ldo
  int ldo;
  float* part;      // kSfEpiPartial: [splits][M][N]
};

__device__ void sf_gemm_phase(const SfParams& p, const SfGemm& g, uint8_t* smem, uint64_t* bars, uint32_t tmem,
                              SfState& st, int* s_fail) {
  const int warp = warp_id();
  const int lane = lane_id();
  uint64_t* full = bars;
  uint64_t* empty = bars + kSfStages;
  uint64_t* accb = bars + 2 * kSfStages;
  const int m_tiles = (g.M + kSfBM - 1) / kSfBM;
  const int n_tiles = g.N / kSfBN;
  const int kbs = g.K / kSfBK;
  const int kps = (kbs + g.splits - 1) / g.splits;
  const int units = m_tiles * n_tiles * g.splits;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int tile = u / g.splits;
    const int sp = u - tile * g.splits;
    const int mt = tile / n_tiles;
    const int nt = tile - mt * n_tiles;
    const int kb_lo = sp * kps;
    const int kb_hi = kb_lo + kps < kbs ? kb_lo + kps : kbs;
    const int nk = kb_hi > kb_lo ? kb_hi - kb_lo : 0;
    if (st.ok && nk > 0) {
      if (warp == 0) {
        if (lane == 0) {
          fence_proxy_async_global();
          for (int i = 0; i < nk; ++i) {
            const int q = st.it + i;
            const int s = q % kSfStages;
            if (!mbar_wait(&empty[s], ((q / kSfStages) & 1) ^ 1, p.status, kDevTimeoutProducer)) {
              *s_fail = 1;
              break;
            }
            uint8_t* sa = smem + s * kSfStageBytes;
            mbar_arrive_expect_tx(&full[s], kSfStageBytes);
            tma_load_2d(sa, g.ma, &full[s], (kb_lo + i) * kSfBK, mt * kSfBM);
            tma_load_2d(sa + kSfABytes, g.mw, &full[s], (kb_lo + i) * kSfBK, nt * kSfBN);
            st.it_issued = q + 1;
          }
        }
      } else if (warp == 1) {
        if (lane == 0) {
          constexpr uint32_t idesc = idesc_f16_f32(kSfBM, kSfBN);
          const uint32_t base = smem_u32(smem);
          for (int i = 0; i < nk; ++i) {
            const int q = st.it + i;
            const int s = q % kSfStages;
            if (!mbar_wait(&full[s], (q / kSfStages) & 1, p.status, kDevTimeoutMma)) {
              *s_fail = 1;
              break;
            }
            tc_fence_after();
            const uint32_t sa = base + s * kSfStageBytes;
            const uint32_t sb = sa + kSfABytes;
#pragma unroll
            for (int k = 0; k < kSfBK / 16; ++k)
              umma_f16_ss(tmem, smem_desc_sw128(sa + k * 32, 16, 1024), smem_desc_sw128(sb + k * 32, 16, 1024),
                          idesc, (i > 0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          umma_commit(accb);  // arrives once every MMA issued so far has completed
        }
      } else if (warp >= 4) {
        const int qtr = warp & 3;
        if (mbar_wait(accb, st.acc & 1, p.status, kDevTimeoutEpilogue)) {
          tc_fence_after();
          uint32_t r[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(qtr * 32) << 16), r);
          tmem_wait_ld();
          const int row = mt * kSfBM + qtr * 32 + lane;
          const int n0 = nt * kSfBN;
          if (row < g.M) {
            if (g.epi == kSfEpiPartial) {
              float4* dst = reinterpret_cast<float4*>(g.part + (static_cast<long long>(sp) * g.M + row) * g.N + n0);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                     __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
            } else {
              uint4* dst = reinterpret_cast<uint4*>(g.out16 + static_cast<long long>(row) * g.ldo + n0);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  v[e] = __uint_as_float(r[8 * i + e]) + __ldg(g.bias + n0 + 8 * i + e);
                  if (g.epi == kSfEpiGelu) v[e] = gelu_erf(v[e]);
                }
                dst[i] = make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]),
                                    pack_half2(v[6], v[7]));
              }
            }
          }
        } else {
          *s_fail = 1;
        }
      }
    }
    if (nk > 0) {
      st.it += nk;
      st.acc += 1;
    }
    tc_fence_before();
    __syncthreads();  // the accumulator and the stages are free for the next unit
    tc_fence_after();
    if (*s_fail) st.ok = false;
  }
}

// ---------------------------------------------------------------------------
// attention phase: one unit per (batch element, head); S <= 128 queries and
// keys, head_dim 64, all in one 128 x 128 block
// ---------------------------------------------------------------------------
__device__ void sf_attention_phase(const SfParams& p, uint8_t* smem, uint64_t* bars, uint32_t tmem, SfState& st,
                                   int* s_fail) {
  const int warp = warp_id();
  const int lane = lane_id();
  uint64_t* attn_in = bars + 2 * kSfStages + 1;
  uint64_t* s_full = attn_in + 1;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = p_full + 1;
  const int units = p.B * p.H;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int b = u / p.H;
    const int h = u - b * p.H;
    const uint32_t par = st.attn & 1;
    if (st.ok) {
      if (warp == 0) {
        if (lane == 0) {
          fence_proxy_async_global();
          mbar_arrive_expect_tx(attn_in, 3 * kSfTileBytes);
          const int y = b * p.S;
          tma_load_2d(smem, &p.a_qkv, attn_in, h * 64, y);
          tma_load_2d(smem + kSfTileBytes, &p.a_qkv, attn_in, p.D + h * 64, y);
          tma_load_2d(smem + 2 * kSfTileBytes, &p.a_qkv, attn_in, 2 * p.D + h * 64, y);
          st.attn_issued = st.attn + 1;
        }
      } else if (warp == 1) {
        if (lane == 0) {
          const uint32_t base = smem_u32(smem);
          constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);
          constexpr uint32_t idesc_o = idesc_f16_f32(128, 64, false, true);  // K-major P, MN-major V
          if (mbar_wait(attn_in, par, p.status, kDevTimeoutMma)) {
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16_ss(tmem, smem_desc_sw128(base + k * 32, 16, 1024),
                          smem_desc_sw128(base + kSfTileBytes + k * 32, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
            umma_commit(s_full);
            if (mbar_wait(p_full, par, p.status, kDevTimeoutMma)) {
              tc_fence_after();
              const uint32_t va = base + 2 * kSfTileBytes;
              // P: 128 keys = 64 TMEM columns, 8 per MMA; V MN-major, 16 keys = 2048 B
#pragma unroll
              for (int k = 0; k < 8; ++k)
                umma_f16_ts(tmem + kSfTmemO, tmem + k * 8, smem_desc_sw128(va + k * 2048, 16384, 1024), idesc_o,
                            k > 0 ? 1u : 0u);
            } else {
              *s_fail = 1;
            }
          } else {
            *s_fail = 1;
          }
          umma_commit(o_full);
        }
      } else if (warp >= 4) {
        const int qtr = warp & 3;
        const int r = qtr * 32 + lane;  // query row within the block
        const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
        float l = 0.f;
        bool good = mbar_wait(s_full, par, p.status, kDevTimeoutSoftmax);
        if (good) {
          tc_fence_after();
          float s[128];
          {
            uint32_t v[128];
            tmem_ld128(tmem + lane_off, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(v[i]);
          }
          // keys of this batch element only (the tile's later rows belong to
          // the next one or lie outside the tensor), causal: key <= query
          const int lim = p.causal ? (r + 1 < p.S ? r + 1 : p.S) : p.S;
          float mx = -INFINITY;
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            s[i] = i < lim ? s[i] : -INFINITY;
            mx = fmaxf(mx, s[i]);
          }
          const float c = p.scale_log2;
          const float m = mx * c;
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
        } else {
          *s_fail = 1;
        }
        tc_fence_before();
        mbar_arrive(p_full);  // always: the MMA thread's wait must not hang on a failed row
        if (good && mbar_wait(o_full, par, p.status, kDevTimeoutSoftmax)) {
          tc_fence_after();
          uint32_t ov[64];
          tmem_ld64(tmem + lane_off + kSfTmemO, ov);
          tmem_wait_ld();
          if (r < p.S) {
            const float inv = 1.f / l;
            uint4* dst = reinterpret_cast<uint4*>(p.ctx + static_cast<long long>(b * p.S + r) * p.D + h * 64);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_uint4(pack_half2(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv),
                                  pack_half2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv),
                                  pack_half2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv),
                                  pack_half2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv));
          }
        } else if (good) {
          *s_fail = 1;
        }
      }
    }
    st.attn += 1;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (*s_fail) st.ok = false;
  }
}

// ---------------------------------------------------------------------------
// row phase: one warp per row; v = (x_in) + bias + sum of the split-K
// partials in split order; optionally stored as the residual; then the
// two-pass LayerNorm of v, stored as fp16 (next GEMM's operand) or fp32
// (the final output). D % 128 == 0, D <= 1024.
// ---------------------------------------------------------------------------
struct SfRows {
  const float* x_in;  // residual source (may equal x_out)
  float* x_out;       // or nullptr
  const float* bias;  // or nullptr (no partials either)
  const float* part;
  int splits;
  const float* w;
  const float* b;
  float eps;
  uint16_t* normed16;  // one of these two
  float* out32;
};

__device__ void sf_rows_phase(const SfParams& p, const SfRows& rw) {
  const int warp = warp_id();
  const int lane = lane_id();
  const int nq = p.D / 128;  // float4 per lane
  const long long plane = static_cast<long long>(p.M) * p.D;
  for (int row = blockIdx.x * (kSfThreads / 32) + warp; row < p.M; row += gridDim.x * (kSfThreads / 32)) {
    float4 v[8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < nq) {
        const int col = 4 * (lane + 32 * i);
        const long long off = static_cast<long long>(row) * p.D + col;
        float4 a = *reinterpret_cast<const float4*>(rw.x_in + off);
        if (rw.bias != nullptr) {
          float4 t = *reinterpret_cast<const float4*>(rw.part + off);
          for (int s = 1; s < rw.splits; ++s) {
            const float4 q = *reinterpret_cast<const float4*>(rw.part + s * plane + off);
            t.x += q.x;
            t.y += q.y;
            t.z += q.z;
            t.w += q.w;
          }
          const float4 bq = __ldg(reinterpret_cast<const float4*>(rw.bias + col));
          a.x += t.x + bq.x;
          a.y += t.y + bq.y;
          a.z += t.z + bq.z;
          a.w += t.w + bq.w;
        }
        if (rw.x_out != nullptr) *reinterpret_cast<float4*>(rw.x_out + off) = a;
        v[i] = a;
        sum += (a.x + a.y) + (a.z + a.w);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(p.D);
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < nq) {
        const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
        sq += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / static_cast<float>(p.D) + rw.eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < nq) {
        const int col = 4 * (lane + 32 * i);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(rw.w + col));
        const float4 bv = __ldg(reinterpret_cast<const float4*>(rw.b + col));
        const float y0 = (v[i].x - mean) * rstd * wv.x + bv.x;
        const float y1 = (v[i].y - mean) * rstd * wv.y + bv.y;
        const float y2 = (v[i].z - mean) * rstd * wv.z + bv.z;
        const float y3 = (v[i].w - mean) * rstd * wv.w + bv.w;
        const long long off = static_cast<long long>(row) * p.D + col;
        if (rw.out32 != nullptr) {
          *reinterpret_cast<float4*>(rw.out32 + off) = make_float4(y0, y1, y2, y3);
        } else {
          *reinterpret_cast<uint2*>(rw.normed16 + off) = make_uint2(pack_half2(y0, y1), pack_half2(y2, y3));
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kSfThreads, 1) small_forward_kernel(const __grid_constant__ SfParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSfBarOff);
  uint64_t* drain = bars + 2 * kSfStages + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kSfNumBars);
  __shared__ int s_fail;
  __shared__ int s_flag;
  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSfNumBars; ++i) mbar_init(&bars[i], i == 2 * kSfStages + 3 ? 128 : 1);  // p_full: 128 rows
    fence_mbar_init();
    s_fail = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kSfTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  SfState st{0, 0, 0, true, 0, 0};

  // norm1 of the first layer
  {
    SfRows rw{p.x, nullptr, nullptr, nullptr, 1, p.layer[0].n1w, p.layer[0].n1b, p.layer[0].eps1, p.normed, nullptr};
    if (st.ok) sf_rows_phase(p, rw);
  }
  st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
  for (int l = 0; l < p.L; ++l) {
    const SfLayer& ly = p.layer[l];
    {
      SfGemm g{&p.a_normed, &p.w[l][0], p.M, 3 * p.D, p.D, 1, kSfEpiBias, ly.bqkv, p.qkv, 3 * p.D, nullptr};
      sf_gemm_phase(p, g, smem, bars, tmem, st, &s_fail);
    }
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    sf_attention_phase(p, smem, bars, tmem, st, &s_fail);
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    {
      SfGemm g{&p.a_ctx, &p.w[l][1], p.M, p.D, p.D, p.sp_o, kSfEpiPartial, nullptr, nullptr, 0, p.ws};
      sf_gemm_phase(p, g, smem, bars, tmem, st, &s_fail);
    }
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    {
      SfRows rw{l == 0 ? p.x : p.xr, p.xr, ly.bo, p.ws, p.sp_o, ly.n2w, ly.n2b, ly.eps2, p.normed, nullptr};
      if (st.ok) sf_rows_phase(p, rw);
    }
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    {
      SfGemm g{&p.a_normed, &p.w[l][2], p.M, p.F, p.D, 1, kSfEpiGelu, ly.b1, p.hidden, p.F, nullptr};
      sf_gemm_phase(p, g, smem, bars, tmem, st, &s_fail);
    }
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    {
      SfGemm g{&p.a_hidden, &p.w[l][3], p.M, p.D, p.F, p.sp_2, kSfEpiPartial, nullptr, nullptr, 0, p.ws};
      sf_gemm_phase(p, g, smem, bars, tmem, st, &s_fail);
    }
    st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
    {
      const bool last = l + 1 == p.L;
      SfRows rw{p.xr, last ? nullptr : p.xr, ly.b2, p.ws, p.sp_2, last ? p.fw : p.layer[l + 1].n1w,
                last ? p.fb : p.layer[l + 1].n1b, last ? p.feps : p.layer[l + 1].eps1, last ? nullptr : p.normed,
                last ? p.out : nullptr};
      if (st.ok) sf_rows_phase(p, rw);
    }
    if (l + 1 < p.L) st.ok = sf_grid_barrier(p.bar, p.status, st.ok, &s_flag) && st.ok;
  }

  // drain: the loads and MMAs this CTA issued have completed before the CTA
  // (and its TMEM) goes away; with every wait successful this is immediate
  if (warp == 0 && lane == 0) {
    const int first = st.it_issued > kSfStages ? st.it_issued - kSfStages : 0;
    for (int q = first; q < st.it_issued; ++q)
      mbar_wait(&bars[q % kSfStages], (q / kSfStages) & 1, nullptr, kDevTimeoutDrain);
    if (st.attn_issued > 0) mbar_wait(&bars[2 * kSfStages + 1], (st.attn_issued - 1) & 1, nullptr, kDevTimeoutDrain);
  }
  if (warp == 1 && lane == 0) {
    umma_commit(drain);
    mbar_wait(drain, 0, nullptr, kDevTimeoutDrain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kSfTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static long long sf_align(long long v) { return (v + 255) & ~255ll; }

// Split count of a split-K phase: about one work unit per SM, at least one
// k-block per unit, no empty split.
static int sf_splits(int tiles, int kbs, int grid) {
  int sp = grid / (tiles > 0 ? tiles : 1);
  if (sp < 1) sp = 1;
  if (sp > kbs) sp = kbs;
  const int kps = (kbs + sp - 1) / sp;
  return (kbs + kps - 1) / kps;
}

struct SfLayout {
  long long normed, qkv, ctx, hidden, xr, ws, bar, total;
};

static SfLayout sf_layout(long long M, long long D, long long F, int max_splits) {
  SfLayout o;
  long long off = 0;
  o.normed = off;
  off = sf_align(off + M * D * 2);
  o.qkv = off;
  off = sf_align(off + M * 3 * D * 2);
  o.ctx = off;
  off = sf_align(off + M * D * 2);
  o.hidden = off;
  off = sf_align(off + M * F * 2);
  o.xr = off;
  off = sf_align(off + M * D * 4);
  o.ws = off;
  off = sf_align(off + static_cast<long long>(max_splits) * M * D * 4);
  o.bar = off;
  off = sf_align(off + 16);
  o.total = off;
  return o;
}

static int sf_grid() {
  static int grid[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (grid[dev & 63] == 0) {
    cudaError_t e = cudaFuncSetAttribute(small_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSfSmemAlloc);
    if (e != cudaSuccess) return -set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(small forward): %s", cudaGetErrorString(e));
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, small_forward_kernel, kSfThreads, kSfSmemAlloc);
    if (e != cudaSuccess || per_sm < 1)
      return -set_error(TF_ERR_LAUNCH, "small forward: no resident CTA per SM (%s)", cudaGetErrorString(e));
    grid[dev & 63] = device_sm_count();  // one CTA per SM
  }
  return grid[dev & 63];
}

static bool sf_shape_ok(long long B, long long S, long long D, long long H, long long F, long long L) {
  return B > 0 && S > 0 && S <= 128 && B * S <= 512 && D > 0 && D % 128 == 0 && D <= 1024 && H > 0 &&
         D == 64 * H && F > 0 && F % kSfBK == 0 && F <= 8192 && L > 0 && L <= kSfMaxLayers;
}

long long forward_small_workspace_bytes(long long B, long long S, long long D, long long F) {
  if (B <= 0 || S <= 0 || D <= 0 || F <= 0) return 0;
  return sf_layout(B * S, D, F, kSfMaxSplits).total;
}

int forward_small(const SmallFwdArgs& a, cudaStream_t stream) {
  const long long B = a.batch, S = a.seq, D = a.d_model, H = a.heads, F = a.ffn, L = a.layers;
  if (!sf_shape_ok(B, S, D, H, F, L))
    return set_error(TF_ERR_SHAPE,
                     "forward_small: B=%lld S=%lld D=%lld H=%lld F=%lld L=%lld (needs S <= 128, B*S <= 512, "
                     "head_dim 64, D %% 128 == 0 and <= 1024, F %% 64 == 0 and <= 8192, L <= %d)",
                     B, S, D, H, F, L, kSfMaxLayers);
  if (a.x == nullptr || a.out == nullptr || a.params == nullptr || a.eps == nullptr || a.workspace == nullptr)
    return set_error(TF_ERR_SHAPE, "forward_small: null argument");
  if (!aligned16(a.x) || !aligned16(a.out) || (reinterpret_cast<uintptr_t>(a.workspace) & 255) != 0)
    return set_error(TF_ERR_ALIGN, "forward_small: x and out 16-byte aligned, workspace 256-byte aligned");
  const long long M = B * S;
  const SfLayout lay = sf_layout(M, D, F, kSfMaxSplits);
  if (a.workspace_bytes < lay.total)
    return set_error(TF_ERR_SHAPE, "forward_small: workspace of %lld bytes needed", lay.total);
  const int grid = sf_grid();
  if (grid <= 0) return -grid;

  SfParams p;
  memset(&p, 0, sizeof(p));
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  p.normed = reinterpret_cast<uint16_t*>(ws + lay.normed);
  p.qkv = reinterpret_cast<uint16_t*>(ws + lay.qkv);
  p.ctx = reinterpret_cast<uint16_t*>(ws + lay.ctx);
  p.hidden = reinterpret_cast<uint16_t*>(ws + lay.hidden);
  p.xr = reinterpret_cast<float*>(ws + lay.xr);
  p.ws = reinterpret_cast<float*>(ws + lay.ws);
  p.bar = reinterpret_cast<unsigned*>(ws + lay.bar);
  p.x = a.x;
  p.out = a.out;
  p.status = device_status_ptr();
  if (p.status == nullptr) return last_error_code();
  int rc = 0;
  if ((rc = make_tmap_2d_f16(&p.a_normed, p.normed, D, M, D, kSfBK, kSfBM))) return rc;
  if ((rc = make_tmap_2d_f16(&p.a_ctx, p.ctx, D, M, D, kSfBK, kSfBM))) return rc;
  if ((rc = make_tmap_2d_f16(&p.a_hidden, p.hidden, F, M, F, kSfBK, kSfBM))) return rc;
  if ((rc = make_tmap_2d_f16(&p.a_qkv, p.qkv, 3 * D, M, 3 * D, 64, 128))) return rc;
  for (int l = 0; l < L; ++l) {
    const void* const* w = a.params + 12 * l;
    for (int i = 0; i < 12; ++i)
      if (w[i] == nullptr || !aligned16(w[i])) return set_error(TF_ERR_ALIGN, "forward_small: layer %d parameter %d", l, i);
    if ((rc = make_tmap_2d_f16(&p.w[l][0], w[0], D, 3 * D, D, kSfBK, kSfBN))) return rc;
    if ((rc = make_tmap_2d_f16(&p.w[l][1], w[2], D, D, D, kSfBK, kSfBN))) return rc;
    if ((rc = make_tmap_2d_f16(&p.w[l][2], w[4], D, F, D, kSfBK, kSfBN))) return rc;
    if ((rc = make_tmap_2d_f16(&p.w[l][3], w[6], F, D, F, kSfBK, kSfBN))) return rc;
    SfLayer& ly = p.layer[l];
    ly.bqkv = static_cast<const float*>(w[1]);
    ly.bo = static_cast<const float*>(w[3]);
    ly.b1 = static_cast<const float*>(w[5]);
    ly.b2 = static_cast<const float*>(w[7]);
    ly.n1w = static_cast<const float*>(w[8]);
    ly.n1b = static_cast<const float*>(w[9]);
    ly.n2w = static_cast<const float*>(w[10]);
    ly.n2b = static_cast<const float*>(w[11]);
    ly.eps1 = a.eps[2 * l];
    ly.eps2 = a.eps[2 * l + 1];
  }
  p.fw = static_cast<const float*>(a.params[12 * L]);
  p.fb = static_cast<const float*>(a.params[12 * L + 1]);
  if (p.fw == nullptr || p.fb == nullptr || !aligned16(p.fw) || !aligned16(p.fb))
    return set_error(TF_ERR_ALIGN, "forward_small: final LayerNorm parameters");
  p.feps = a.eps[2 * L];
  p.scale_log2 = 0.125f * 1.4426950408889634f;  // head_dim 64
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.D = static_cast<int>(D);
  p.H = static_cast<int>(H);
  p.F = static_cast<int>(F);
  p.L = static_cast<int>(L);
  p.M = static_cast<int>(M);
  p.causal = a.causal ? 1 : 0;
  const int m_tiles = static_cast<int>((M + kSfBM - 1) / kSfBM);
  const int n_tiles = static_cast<int>(D / kSfBN);
  p.sp_o = sf_splits(m_tiles * n_tiles, static_cast<int>(D / kSfBK), grid);
  p.sp_2 = sf_splits(m_tiles * n_tiles, static_cast<int>(F / kSfBK), grid);
  if (p.sp_o > kSfMaxSplits || p.sp_2 > kSfMaxSplits) return set_error(TF_ERR_SHAPE, "forward_small: split plan");

  cudaError_t e = cudaMemsetAsync(p.bar, 0, 8, stream);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "forward_small: barrier reset: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSfThreads);
  cfg.dynamicSmemBytes = kSfSmemAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, small_forward_kernel, p);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "forward_small launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
