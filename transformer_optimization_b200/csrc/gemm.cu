// 16-bit GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] = epilogue( A[M,K] · W[N,K]^T + bias[N] )   (A, W, C fp16 or bf16)
//
// This is the projection the reference runs four times per layer on its
// fp32-model fast path (packed QKV, out_proj, ffn_in+GELU, ffn_out:
// torch_transformer_benchmark.py:4138-4194, Triton kernel 1756-1803).
// Epilogues (all on the fp32 accumulator plus an fp32 bias):
//   EPI 0  C = fp16(acc + bias)
//   EPI 1  C = fp16(gelu_erf(acc + bias))        erf GELU in fp32 (A&S 7.1.28 erf)
//   EPI 2  x_out = mask_x(x_in + mask_delta(acc + bias))   fp32 residual
// EPI 2 is the residual add of the reference's next LayerNorm site
// (torch_transformer_benchmark.py:3988-3995) moved into the GEMM, with the
// same two masking points. Compared with the reference's fp16 fast path this
// drops three fp16 roundings (bias, GELU input, residual delta); the result
// is closer to the fp32 eager model the accuracy gate compares against.
// The half-precision models (fp16 or bf16 parameters and activations, type
// T) keep the roundings of their eager forward (torch_transformer_benchmark.py:
// 162-224 run in T), where every op stores a T tensor:
//   EPI 4  x_out = T(mask_x(x_in + mask_delta(T(acc + bias))))   residual in T
//   EPI 5  C = T(gelu_erf(T(acc + bias)))        F.gelu of the stored Linear
// The operand type (and C's) is the template parameter DT.
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
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle row of fp16
constexpr int kGemmThreads = 192;
constexpr int kEpiTileFloats = 32 * 32;  // one warp's epilogue staging tile (32 x 32 fp32)
constexpr int kMaxSplits = 32;           // split-K: most k ranges per tile
// k-blocks per stage group: the MMA thread waits once and commits once per
// group. Every barrier wait and commit of the issuing thread leaves the tensor
// pipe idle for a while (its MMA queue is shallow); measured on B200 with the
// c3 forward (alternating on one box, 3 runs each): 1 k-block 7.95 ms, 2
// k-blocks 7.82 ms (GEMMs 1120 -> 1145 TFLOP/s in the step); 3 k-blocks per
// group (two groups of the 2-SM kernel's six stages) was slower than 1.
constexpr int kGemmGroupKb = 2;

struct GemmArgs {
  const float* bias;
  uint16_t* C;  // EPI 0/1/5: fp16 or bf16 elements
  long long ldc;
  const float* x_in;  // EPI 2
  float* x_out;
  const uint16_t* x16_in;  // EPI 4: residual in the operand type
  uint16_t* x16_out;
  long long ldx;
  const uint8_t* valid;
  int mask_mode;  // EPI 2/4: 0 none, 1 mask_delta, 2 mask_x
  int M, N, K;    // K: columns of A
  int a_repeat;   // 1, or 2 for split weights (W has a_repeat*K columns)
  int m_tiles, n_tiles;
  int* status;
  // split-K (EPI 3): each tile's k-blocks are cut into `splits` ranges of
  // kb_per_split; work unit u = tile * splits + split; the fp32 partial of a
  // unit goes to ws[split][M][N]. splits = 1 otherwise.
  int splits, kb_per_split;
  float* ws;
  // EPI 2/4, optional: per 8-row group, the count of x_out columns stored so
  // far (a group is complete at N); read by a LayerNorm that runs alongside
  int* ready;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;  // 4 warps x 32x33 floats
  static constexpr int kBarOffset = kEpiOffset + 4 * kEpiTileFloats * 4;
  // full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, tmem slot
  static constexpr int kBytes = kBarOffset + (2 * STAGES + 5) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

// L2 prefetch of this warp's residual rows for a whole tile (EPI 2, 4): lane
// L touches row row0 + L, `width` columns from col0, one 128-byte line at a
// time. Issued before the warp waits for the tile's accumulator, so the HBM
// reads overlap the tile's main loop and the register loads below hit L2.
template <int EPI>
__device__ __forceinline__ void prefetch_residual_l2(const GemmArgs& p, int row0, int col0, int width) {
  const int row = row0 + (threadIdx.x & 31);
  if (row >= p.M) return;
  constexpr int kLine = EPI == 4 ? 64 : 32;  // elements per 128-byte line
  const char* base = EPI == 4 ? reinterpret_cast<const char*>(p.x16_in + static_cast<long long>(row) * p.ldx)
                              : reinterpret_cast<const char*>(p.x_in + static_cast<long long>(row) * p.ldx);
  for (int c = col0; c < col0 + width && c < p.N; c += kLine)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + static_cast<long long>(c) * (EPI == 4 ? 2 : 4)));
}

// Residual rows of one chunk for this lane (EPI 2, 4): rows row0 + it*4 +
// L/8, columns col0 + 4*(L%8), it = 0..7, widened to fp32 (exact). Issued
// ahead of use so the HBM latency overlaps the previous chunk.
template <int EPI, int DT>
__device__ __forceinline__ void load_residual(const GemmArgs& p, float4 (&xv)[8], int row0, int col0) {
  const int lane = threadIdx.x & 31;
  const int c4 = (lane & 7) * 4;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int row = row0 + it * 4 + (lane >> 3);
    if (row >= p.M) {
      xv[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if constexpr (EPI == 4) {
      const uint2 h = __ldcs(reinterpret_cast<const uint2*>(p.x16_in + static_cast<long long>(row) * p.ldx + col0 + c4));
      const float2 a = unpack2<DT>(h.x), b = unpack2<DT>(h.y);
      xv[it] = make_float4(a.x, a.y, b.x, b.y);
    } else {
      xv[it] = __ldcs(reinterpret_cast<const float4*>(p.x_in + static_cast<long long>(row) * p.ldx + col0 + c4));
    }
  }
}

// Epilogue of one 32-row x 32-column accumulator chunk, cooperatively by the
// warp that read it from TMEM (lane i holds row row0+i). The chunk is staged
// through a 32 x 32 float shared-memory tile (16-byte chunks XOR-swizzled by
// row, conflict-free both ways) so that the global accesses run along rows:
// lane L handles columns 4*(L%8)..+3 of rows it*4 + L/8, i.e. each store
// instruction covers 4 rows x 64 B (16-bit) or 4 rows x 128 B (fp32) instead
// of 32 scattered rows.
template <int EPI, int DT>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& p, const uint32_t (&r)[32], float* buf, int row0,
                                               int col0, const float4 (&xv)[8], int split = 0) {
  const int lane = threadIdx.x & 31;
  // 16-byte chunk c of row r sits at chunk c ^ (r % 8) of the row's 128 bytes:
  // both the row-wise writes (lanes = rows) and the column-wise reads below
  // (8 lanes = one row's 8 chunks) touch 8 different chunks per quarter-warp,
  // so the vector accesses are free of bank conflicts without padding
  float4* tile = reinterpret_cast<float4*>(buf);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    tile[lane * 8 + (c ^ (lane & 7))] = make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                                    __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
  __syncwarp();
  const int c4 = (lane & 7) * 4;
  const float4 bq = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + c4));
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rl = it * 4 + (lane >> 3);
    const int row = row0 + rl;
    const float4 a = tile[rl * 8 + ((lane & 7) ^ (rl & 7))];
    const float src[4] = {a.x, a.y, a.z, a.w};
    if constexpr (EPI == 3) {
      // split-K partial: the raw fp32 sum of this unit's k-blocks (no bias)
      if (row < p.M)
        *reinterpret_cast<float4*>(p.ws + (static_cast<long long>(split) * p.M + row) * p.N + col0 + c4) =
            make_float4(src[0], src[1], src[2], src[3]);
      continue;
    }
    float v0 = src[0] + bq.x, v1 = src[1] + bq.y, v2 = src[2] + bq.z, v3 = src[3] + bq.w;
    if (row < p.M) {
      if constexpr (EPI == 2) {
        const long long off = static_cast<long long>(row) * p.ldx + col0 + c4;
        bool valid = true;
        if (p.mask_mode != 0) valid = p.valid[row] != 0;
        if (p.mask_mode == 1 && !valid) v0 = v1 = v2 = v3 = 0.f;
        float4 o = make_float4(xv[it].x + v0, xv[it].y + v1, xv[it].z + v2, xv[it].w + v3);
        if (p.mask_mode == 2 && !valid) o = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(p.x_out + off) = o;
      } else if constexpr (EPI == 4) {
        // the Linear's output is stored in T before the add; the sum is
        // rounded to T again by the store
        const long long off = static_cast<long long>(row) * p.ldx + col0 + c4;
        bool valid = true;
        if (p.mask_mode != 0) valid = p.valid[row] != 0;
        v0 = round16<DT>(v0);
        v1 = round16<DT>(v1);
        v2 = round16<DT>(v2);
        v3 = round16<DT>(v3);
        if (p.mask_mode == 1 && !valid) v0 = v1 = v2 = v3 = 0.f;
        float4 o = make_float4(xv[it].x + v0, xv[it].y + v1, xv[it].z + v2, xv[it].w + v3);
        if (p.mask_mode == 2 && !valid) o = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<uint2*>(p.x16_out + off) = make_uint2(pack2<DT>(o.x, o.y), pack2<DT>(o.z, o.w));
      } else {
        if constexpr (EPI == 1) {
          v0 = gelu_erf(v0);
          v1 = gelu_erf(v1);
          v2 = gelu_erf(v2);
          v3 = gelu_erf(v3);
        } else if constexpr (EPI == 5) {
          v0 = gelu_erf(round16<DT>(v0));
          v1 = gelu_erf(round16<DT>(v1));
          v2 = gelu_erf(round16<DT>(v2));
          v3 = gelu_erf(round16<DT>(v3));
        }
        *reinterpret_cast<uint2*>(p.C + static_cast<long long>(row) * p.ldc + col0 + c4) =
            make_uint2(pack2<DT>(v0, v1), pack2<DT>(v2, v3));
      }
    }
  }
  __syncwarp();  // the tile is reused by the next chunk
}

// residual epilogues (the accumulator is added to rows of x)
template <int EPI>
constexpr bool kResidualEpi = EPI == 2 || EPI == 4;

// After a warp has stored its rows row0..row0+31 of a tile (`cols` columns of
// x_out): add `cols` to the ready counts of the four 8-row groups. Every lane
// fences its own stores; the counts are release adds, so a reader that
// acquires a complete count sees every column of the group.
__device__ __forceinline__ void signal_rows(const GemmArgs& p, int row0, int cols) {
  __threadfence();
  __syncwarp();
  const int lane = threadIdx.x & 31;
  if (lane < 4 && cols > 0) {
    const int r = row0 + lane * 8;
    if (r < p.M) red_release_gpu_add(p.ready + (r >> 3), cols);
  }
}

template <int BN, int STAGES, int EPI, int DT, int KG>
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
  // work units: (tile, split) with the k-block range [kb_lo, kb_hi)
  const int total_units = total_tiles * p.splits;
  auto unit_range = [&](int u, int& tile, int& sp, int& kb_lo, int& kb_hi) {
    tile = u / p.splits;
    sp = u - tile * p.splits;
    kb_lo = sp * p.kb_per_split;
    kb_hi = kb_lo + p.kb_per_split < k_blocks ? kb_lo + p.kb_per_split : k_blocks;
  };

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
  // everything above touched only this CTA's shared memory and TMEM
  pdl_wait();
  pdl_trigger();

  // Stages are filled and consumed in groups of KG k-blocks: one `full` wait
  // and one commit per group (kGemmGroupKb). Group barrier g covers stages
  // KG*g .. KG*g+KG-1.
  constexpr int kGroups = STAGES / KG;
  static_assert(STAGES % KG == 0, "stages are used in groups of KG");
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int ig = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int t, sp, kb_lo, kb_hi;
        unit_range(u, t, sp, kb_lo, kb_hi);
        const int m0 = (t / p.n_tiles) * kGemmBM;
        const int n0 = (t % p.n_tiles) * BN;
        for (int kg = kb_lo; kg < kb_hi; kg += KG, ++ig) {
          const int sg = ig % kGroups;
          const uint32_t ph = (ig / kGroups) & 1;
          if (!mbar_wait(&empty[sg], ph ^ 1, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const int nkb = kb_hi - kg < KG ? kb_hi - kg : KG;
          mbar_arrive_expect_tx(&full[sg], nkb * L::kStageBytes);
          for (int j = 0; j < nkb; ++j) {
            const int kb = kg + j;
            uint8_t* sa = smem + (KG * sg + j) * L::kStageBytes;
            const int akb = kb < a_blocks ? kb : kb - a_blocks;
            tma_load_2d(sa, &tmA, &full[sg], akb * kGemmBK, m0);
            // W block: columns [kb*64, kb*64+64) of [W_hi | W_lo]; with a
            // K tail the lo half starts at column K, not at a_blocks*64
            const int wcol = kb < a_blocks ? kb * kGemmBK : p.K + akb * kGemmBK;
            tma_load_2d(sa + L::kABytes, &tmB, &full[sg], wcol, n0);
          }
        }
      }
      // Drain: every load this thread issued must land before the CTA exits.
      const int first = ig > kGroups ? ig - kGroups : 0;
      for (int j = first; j < ig; ++j)
        mbar_wait(&full[j % kGroups], (j / kGroups) & 1, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_16_f32(DT, kGemmBM, BN);
      const uint32_t smem_base = smem_u32(smem);
      int ig = 0;
      int tc = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++tc) {
        int t, sp, kb_lo, kb_hi;
        unit_range(u, t, sp, kb_lo, kb_hi);
        const int a = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int kg = kb_lo; kg < kb_hi; kg += KG, ++ig) {
          const int sg = ig % kGroups;
          const uint32_t ph = (ig / kGroups) & 1;
          if (!mbar_wait(&full[sg], ph, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = kb_hi - kg < KG ? kb_hi - kg : KG;
          for (int j = 0; j < nkb; ++j) {
            const uint32_t sa = smem_base + (KG * sg + j) * L::kStageBytes;
            const uint32_t sb = sa + L::kABytes;
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
              const uint64_t ad = smem_desc_sw128(sa + k * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(sb + k * 32, 16, 1024);
              umma_f16_ss(d_tmem, ad, bd, idesc, (kg != kb_lo || j != 0 || k != 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[sg]);
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
    float* ebuf = reinterpret_cast<float*>(smem + L::kEpiOffset) + (warp - 2) * kEpiTileFloats;
    int tc = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++tc) {
      int t, sp, kb_lo, kb_hi;
      unit_range(u, t, sp, kb_lo, kb_hi);
      const int m0 = (t / p.n_tiles) * kGemmBM;
      const int n0 = (t % p.n_tiles) * BN;
      const int a = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      const int row0 = m0 + quarter * 32;
      if constexpr (kResidualEpi<EPI>) prefetch_residual_l2<EPI>(p, row0, n0, BN);
      if (!mbar_wait(&tfull[a], aph, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
      float4 xa[8], xb[8];
      if constexpr (kResidualEpi<EPI>) {
        if (row0 < p.M) load_residual<EPI, DT>(p, xa, row0, n0);
      }
      uint32_t r0[32], r1[32];
      tmem_ld32(t_addr, r0);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        tmem_wait_ld();
        uint32_t(&cur)[32] = (c & 1) ? r1 : r0;
        uint32_t(&nxt)[32] = (c & 1) ? r0 : r1;
        float4(&xcur)[8] = (c & 1) ? xb : xa;
        float4(&xnxt)[8] = (c & 1) ? xa : xb;
        if (c + 1 < BN / 32) {
          tmem_ld32(t_addr + (c + 1) * 32, nxt);
          if constexpr (kResidualEpi<EPI>) {
            if (row0 < p.M && n0 + (c + 1) * 32 < p.N) load_residual<EPI, DT>(p, xnxt, row0, n0 + (c + 1) * 32);
          }
        } else {
          // accumulator fully read: hand the buffer back to the MMA warp
          tc_fence_before();
          mbar_arrive(&tempty[a]);
        }
        const int col0 = n0 + c * 32;
        if (col0 < p.N && row0 < p.M) epilogue_chunk<EPI, DT>(p, cur, ebuf, row0, col0, xcur, sp);
      }
      if constexpr (kResidualEpi<EPI>) {
        if (p.ready != nullptr && row0 < p.M) signal_rows(p, row0, p.N - n0 < BN ? p.N - n0 : BN);
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
// 2-SM variant: a CTA pair (cluster of 2) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2. Each CTA loads its 128 rows of A and half of the
// tile's BN rows of W, so per SM the operand traffic per flop drops by a
// third against the 1-CTA 128 x BN tile and six stages fit in shared memory.
// The leader CTA (rank 0) issues the MMAs; its commits arrive on the
// barriers of both CTAs; both CTAs run the epilogue on their own 128 rows.
//   warp 0      TMA producer (both CTAs, transaction bytes on the leader)
//   warp 1      TMEM allocator (both), MMA issuer (leader)
//   warps 2..9  epilogue: two warpgroups, each half of the BN columns
// ---------------------------------------------------------------------------
constexpr int kGemm2Threads = 320;

template <int BN, int STAGES>
struct Gemm2Smem {
  static constexpr int kABytes = 128 * kGemmBK * 2;       // 16 KB: this CTA's A rows
  static constexpr int kBBytes = (BN / 2) * kGemmBK * 2;  // this CTA's half of W
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;  // 8 warps x 32x33 floats
  static constexpr int kBarOffset = kEpiOffset + 8 * kEpiTileFloats * 4;
  static constexpr int kBytes = kBarOffset + (2 * STAGES + 5) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

template <int BN, int STAGES, int EPI, int DT, int KG>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemm2Threads, 1)
    gemm_f16_tcgen05_2sm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         GemmArgs p) {
  using L = Gemm2Smem<BN, STAGES>;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;
  const int total_tiles = p.m_tiles * p.n_tiles;  // m_tiles counts 256-row tiles here
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
      mbar_init(&tempty[a], 16);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above touched only this CTA's shared memory and TMEM
  pdl_wait();
  pdl_trigger();

  // Stages are filled and consumed in groups of KG k-blocks (kGemmGroupKb):
  // one `full` wait and one commit per group. Group barrier g covers stages
  // KG*g .. KG*g+KG-1.
  constexpr int kGroups = STAGES / KG;
  static_assert(STAGES % KG == 0, "stages are used in groups of KG");
  const int k_groups = (k_blocks + KG - 1) / KG;
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int ig = 0;
      bool ok = true;
      for (int t = cluster_id; t < total_tiles && ok; t += n_clusters) {
        const int m0 = (t / p.n_tiles) * 256 + static_cast<int>(rank) * 128;
        const int n0 = (t % p.n_tiles) * BN + static_cast<int>(rank) * (BN / 2);
        for (int g = 0; g < k_groups; ++g, ++ig) {
          const int sg = ig % kGroups;
          const uint32_t ph = (ig / kGroups) & 1;
          if (!mbar_wait(&empty[sg], ph ^ 1, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const int nkb = k_blocks - KG * g < KG ? k_blocks - KG * g : KG;
          const uint32_t bar = mapa_shared(smem_u32(&full[sg]), 0);
          if (leader) mbar_arrive_expect_tx(&full[sg], nkb * 2 * L::kStageBytes);
          for (int j = 0; j < nkb; ++j) {
            const int kb = KG * g + j;
            uint8_t* sa = smem + (KG * sg + j) * L::kStageBytes;
            const int akb = kb < a_blocks ? kb : kb - a_blocks;
            const int wcol = kb < a_blocks ? kb * kGemmBK : p.K + akb * kGemmBK;
            tma_load_2d_pair(sa, &tmA, bar, akb * kGemmBK, m0);
            tma_load_2d_pair(sa + L::kABytes, &tmB, bar, wcol, n0);
          }
        }
      }
      // Drain: wait until the MMAs have consumed every stage this CTA loaded
      // (the commit that frees a group also proves its loads landed).
      const int first = ig > kGroups ? ig - kGroups : 0;
      for (int j = first; j < ig; ++j)
        mbar_wait(&empty[j % kGroups], ((j / kGroups) & 1), p.status, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader) ----------------
      constexpr uint32_t idesc = idesc_16_f32(DT, 256, BN);
      const uint32_t smem_base = smem_u32(smem);
      int ig = 0;
      int tc = 0;
      bool ok = true;
      for (int t = cluster_id; t < total_tiles && ok; t += n_clusters, ++tc) {
        const int a = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int g = 0; g < k_groups; ++g, ++ig) {
          const int sg = ig % kGroups;
          const uint32_t ph = (ig / kGroups) & 1;
          if (!mbar_wait(&full[sg], ph, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = k_blocks - KG * g < KG ? k_blocks - KG * g : KG;
          for (int j = 0; j < nkb; ++j) {
            const uint32_t sa = smem_base + (KG * sg + j) * L::kStageBytes;
            const uint32_t sb = sa + L::kABytes;
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k)
              umma_f16_ss_pair(d_tmem, smem_desc_sw128(sa + k * 32, 16, 1024),
                               smem_desc_sw128(sb + k * 32, 16, 1024), idesc, (g | j | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[sg], 0x3);
        }
        if (ok) umma_commit_pair_mc(&tfull[a], 0x3);
      }
      umma_commit_pair_mc(drain, 0x1);
      mbar_wait(drain, 0, p.status, kDevTimeoutDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int ew = warp - 2;
    const int half = ew >> 2;       // which half of the BN columns
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    float* ebuf = reinterpret_cast<float*>(smem + L::kEpiOffset) + ew * kEpiTileFloats;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    int tc = 0;
    for (int t = cluster_id; t < total_tiles; t += n_clusters, ++tc) {
      const int m0 = (t / p.n_tiles) * 256 + static_cast<int>(rank) * 128;
      const int n0 = (t % p.n_tiles) * BN + half * (BN / 2);
      const int a = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      const int row0 = m0 + quarter * 32;
      if constexpr (kResidualEpi<EPI>) prefetch_residual_l2<EPI>(p, row0, n0, BN / 2);
      if (!mbar_wait(&tfull[a], aph, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN + half * (BN / 2);
      constexpr int NCH = BN / 64;  // 32-column chunks per half
      float4 xa[8], xb[8];
      if constexpr (kResidualEpi<EPI>) {
        if (row0 < p.M) load_residual<EPI, DT>(p, xa, row0, n0);
      }
      uint32_t r0[32], r1[32];
      tmem_ld32(t_addr, r0);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        tmem_wait_ld();
        uint32_t(&cur)[32] = (c & 1) ? r1 : r0;
        uint32_t(&nxt)[32] = (c & 1) ? r0 : r1;
        float4(&xcur)[8] = (c & 1) ? xb : xa;
        float4(&xnxt)[8] = (c & 1) ? xa : xb;
        if (c + 1 < NCH) {
          tmem_ld32(t_addr + (c + 1) * 32, nxt);
          if constexpr (kResidualEpi<EPI>) {
            if (row0 < p.M && n0 + (c + 1) * 32 < p.N) load_residual<EPI, DT>(p, xnxt, row0, n0 + (c + 1) * 32);
          }
        } else {
          // accumulator fully read: hand the buffer back to the leader's MMA
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader + a * 8);
        }
        const int col0 = n0 + c * 32;
        if (col0 < p.N && row0 < p.M) epilogue_chunk<EPI, DT>(p, cur, ebuf, row0, col0, xcur);
      }
      if constexpr (kResidualEpi<EPI>) {
        if (p.ready != nullptr && row0 < p.M) signal_rows(p, row0, p.N - n0 < BN / 2 ? p.N - n0 : BN / 2);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while its pair may still touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int BN, int STAGES, int EPI, int DT>
static int launch_gemm_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                           cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_f16_tcgen05<BN, STAGES, EPI, DT, kGemmGroupKb>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(gemm): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  cudaError_t e = launch_k(kern, dim3(grid), dim3(kGemmThreads), L::kAlloc, stream, ta, tb, args);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "gemm launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

template <int BN, int STAGES, int EPI, int DT>
static int launch_gemm2_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                            cudaStream_t stream) {
  using L = Gemm2Smem<BN, STAGES>;
  auto kern = gemm_f16_tcgen05_2sm<BN, STAGES, EPI, DT, kGemmGroupKb>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(gemm2): %s", cudaGetErrorString(e));
    attr_done[dev & 63] = true;
  }
  cudaError_t e = launch_k(kern, dim3(grid), dim3(kGemm2Threads), L::kAlloc, stream, ta, tb, args);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "gemm2 launch: %s", cudaGetErrorString(e));
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

// Kernel arguments common to the unsplit and split-K forms.
static GemmArgs make_args(const GemmCall& g) {
  GemmArgs args = {};
  args.bias = g.bias;
  args.C = static_cast<uint16_t*>(g.C);
  args.ldc = g.ldc;
  if (g.epilogue == 4) {
    args.x16_in = static_cast<const uint16_t*>(g.x_in);
    args.x16_out = static_cast<uint16_t*>(g.x_out);
  } else {
    args.x_in = static_cast<const float*>(g.x_in);
    args.x_out = static_cast<float*>(g.x_out);
  }
  args.ldx = g.ldx;
  args.valid = g.valid;
  args.mask_mode = (g.epilogue == 2 || g.epilogue == 4) ? g.mask_mode : 0;
  args.ready = (g.epilogue == 2 || g.epilogue == 4) ? g.ready : nullptr;
  args.M = static_cast<int>(g.M);
  args.N = static_cast<int>(g.N);
  args.K = static_cast<int>(g.K);
  return args;
}

// One instantiation per (epilogue, operand type) of a tiling.
template <int BN, int ST, bool PAIR>
static int launch_by_epi(int epi, int dt, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args,
                         int grid, cudaStream_t stream) {
#define TFB_GEMM_CASE(E, D)                                                          \
  case E * 2 + D:                                                                    \
    if constexpr (PAIR) {                                                            \
      return launch_gemm2_cfg<BN, ST, E, D>(ta, tb, args, grid, stream);             \
    } else {                                                                         \
      return launch_gemm_cfg<BN, ST, E, D>(ta, tb, args, grid, stream);              \
    }
  switch (epi * 2 + dt) {
    TFB_GEMM_CASE(0, 0)
    TFB_GEMM_CASE(1, 0)
    TFB_GEMM_CASE(2, 0)
    TFB_GEMM_CASE(4, 0)
    TFB_GEMM_CASE(5, 0)
    TFB_GEMM_CASE(0, 1)
    TFB_GEMM_CASE(1, 1)
    TFB_GEMM_CASE(2, 1)
    TFB_GEMM_CASE(4, 1)
    TFB_GEMM_CASE(5, 1)
    default: return set_error(TF_ERR_SHAPE, "gemm: epilogue %d with operand type %d", epi, dt);
  }
#undef TFB_GEMM_CASE
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
  if (g.dtype != kDtF16 && g.dtype != kDtBF16) return set_error(TF_ERR_SHAPE, "gemm: operand type %d", g.dtype);
  if (g.epilogue == 0 || g.epilogue == 1 || g.epilogue == 5) {
    if (g.C == nullptr || !aligned16(g.C) || g.ldc % 8 != 0 || g.ldc < N)
      return set_error(TF_ERR_ALIGN, "gemm: C must be 16-byte aligned with a pitch >= N, multiple of 8");
  } else if (g.epilogue == 2 || g.epilogue == 4) {
    const int mult = g.epilogue == 2 ? 4 : 8;  // 16-byte row starts
    if (g.x_in == nullptr || g.x_out == nullptr || !aligned16(g.x_in) || !aligned16(g.x_out) || g.ldx % mult != 0 ||
        g.ldx < N)
      return set_error(TF_ERR_ALIGN, "gemm: residual x must be 16-byte aligned with a pitch >= N, multiple of %d",
                       mult);
    if (g.mask_mode < 0 || g.mask_mode > 2) return set_error(TF_ERR_SHAPE, "gemm: mask mode %d", g.mask_mode);
    if (g.mask_mode != 0 && g.valid == nullptr) return set_error(TF_ERR_SHAPE, "gemm: mask without valid rows");
  } else {
    return set_error(TF_ERR_SHAPE, "gemm: unknown epilogue %d", g.epilogue);
  }

  const int sms = device_sm_count();
  const int m_tiles = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  int bn = g.tile_n > 0 ? g.tile_n : choose_bn(m_tiles, static_cast<int>(N), sms);
  if (N % bn != 0) bn = (N % 128 == 0) ? 128 : 64;
  // 2-SM pairs once 128-wide pair tiles keep at least 4/5 of the CTA pairs
  // busy; 1-CTA tiles (more of them) for smaller problems. Measured at the
  // per-rank c3 shapes of 4 and 8 GPUs: 2048 x 1024 x 4096 with residual
  // 27.9 -> 26.0 us, 4096 x 1024 x 1024 with residual 19.2 -> 15.1 us.
  bool pair = false;
  if (g.pair == 2) {
    pair = true;
  } else if (g.pair == 0) {
    const long long pair_tiles128 = ((M + 255) / 256) * (N / 128);
    pair = (N % 128 == 0) && pair_tiles128 * 5 >= static_cast<long long>(sms / 2) * 4;
  }
  if (pair) {
    if (N % 128 != 0) return set_error(TF_ERR_SHAPE, "gemm: 2-SM tiles need N %% 128 == 0");
    bn = (g.tile_n == 128 || N % 256 != 0) ? 128 : 256;
    if (g.tile_n == 0 && bn == 256) {
      // wave quantisation: prefer 128-wide pair tiles when they fill the
      // device in fewer weighted waves; a 128-wide pair tile costs ~0.82 of
      // a 256-wide one at K = 1024 (measured: 2048 x 3072 x 1024 takes
      // 16.6 us in two waves of 256-wide tiles, 20.4 us in three of 128)
      const long long mt = (M + 255) / 256;
      const long long c256 = mt * (N / 256), c128 = mt * (N / 128);
      const int nc = sms / 2;
      if (0.82 * double((c128 + nc - 1) / nc) < double((c256 + nc - 1) / nc)) bn = 128;
    }
  }

  CUtensorMap ta, tb;
  int rc = make_tmap_2d_f16(&ta, g.A, K, M, g.lda, kGemmBK, 128);
  if (rc) return rc;
  rc = make_tmap_2d_f16(&tb, g.W, K * g.a_repeat, N, g.ldw, kGemmBK, pair ? bn / 2 : bn);
  if (rc) return rc;

  GemmArgs args = make_args(g);
  args.a_repeat = g.a_repeat;
  args.m_tiles = pair ? static_cast<int>((M + 255) / 256) : m_tiles;
  args.n_tiles = static_cast<int>((N + bn - 1) / bn);
  args.status = device_status_ptr();
  if (args.status == nullptr) return last_error_code();
  args.splits = 1;
  args.kb_per_split = static_cast<int>((K + kGemmBK - 1) / kGemmBK) * g.a_repeat;
  args.ws = nullptr;
  const long long tiles = static_cast<long long>(args.m_tiles) * args.n_tiles;
  if (pair) {
    const int max_clusters = sms / 2;
    const int clusters = static_cast<int>(tiles < max_clusters ? tiles : max_clusters);
    const int grid2 = 2 * clusters;
    if (bn == 256) return launch_by_epi<256, 6, true>(g.epilogue, g.dtype, ta, tb, args, grid2, stream);
    return launch_by_epi<128, 8, true>(g.epilogue, g.dtype, ta, tb, args, grid2, stream);
  }
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (bn == 256) return launch_by_epi<256, 4, false>(g.epilogue, g.dtype, ta, tb, args, grid, stream);
  if (bn == 128) return launch_by_epi<128, 6, false>(g.epilogue, g.dtype, ta, tb, args, grid, stream);
  return launch_by_epi<64, 8, false>(g.epilogue, g.dtype, ta, tb, args, grid, stream);
}

// ---------------------------------------------------------------------------
// Split-K for few-row problems: the k-blocks of every 128 x 64 tile are cut
// into `splits` ranges so that tiles x splits CTAs share the work; each unit
// stores its fp32 partial into the workspace ([splits][M][N]), then a second
// kernel sums the partials in fixed split order (deterministic), adds the
// bias and applies the epilogue (16-bit out, GELU, or a residual add).
// ---------------------------------------------------------------------------
template <int EPI, int DT>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmArgs p) {
  pdl_wait();
  pdl_trigger();
  const int nq = p.N >> 2;  // float4 per row
  const long long total = static_cast<long long>(p.M) * nq;
  const long long plane = static_cast<long long>(p.M) * p.N;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / nq);
    const int c = static_cast<int>(i - static_cast<long long>(row) * nq) * 4;
    const float* src = p.ws + static_cast<long long>(row) * p.N + c;
    float4 a = *reinterpret_cast<const float4*>(src);
    for (int sp = 1; sp < p.splits; ++sp) {
      const float4 b = *reinterpret_cast<const float4*>(src + sp * plane);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    const float4 bq = __ldg(reinterpret_cast<const float4*>(p.bias + c));
    float v0 = a.x + bq.x, v1 = a.y + bq.y, v2 = a.z + bq.z, v3 = a.w + bq.w;
    if constexpr (EPI == 2) {
      const long long off = static_cast<long long>(row) * p.ldx + c;
      bool valid = true;
      if (p.mask_mode != 0) valid = p.valid[row] != 0;
      if (p.mask_mode == 1 && !valid) v0 = v1 = v2 = v3 = 0.f;
      const float4 x = *reinterpret_cast<const float4*>(p.x_in + off);
      float4 o = make_float4(x.x + v0, x.y + v1, x.z + v2, x.w + v3);
      if (p.mask_mode == 2 && !valid) o = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(p.x_out + off) = o;
    } else if constexpr (EPI == 4) {
      const long long off = static_cast<long long>(row) * p.ldx + c;
      bool valid = true;
      if (p.mask_mode != 0) valid = p.valid[row] != 0;
      v0 = round16<DT>(v0);
      v1 = round16<DT>(v1);
      v2 = round16<DT>(v2);
      v3 = round16<DT>(v3);
      if (p.mask_mode == 1 && !valid) v0 = v1 = v2 = v3 = 0.f;
      const uint2 h = *reinterpret_cast<const uint2*>(p.x16_in + off);
      const float2 xa = unpack2<DT>(h.x), xb = unpack2<DT>(h.y);
      float4 o = make_float4(xa.x + v0, xa.y + v1, xb.x + v2, xb.y + v3);
      if (p.mask_mode == 2 && !valid) o = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<uint2*>(p.x16_out + off) = make_uint2(pack2<DT>(o.x, o.y), pack2<DT>(o.z, o.w));
    } else {
      if constexpr (EPI == 1) {
        v0 = gelu_erf(v0);
        v1 = gelu_erf(v1);
        v2 = gelu_erf(v2);
        v3 = gelu_erf(v3);
      } else if constexpr (EPI == 5) {
        v0 = gelu_erf(round16<DT>(v0));
        v1 = gelu_erf(round16<DT>(v1));
        v2 = gelu_erf(round16<DT>(v2));
        v3 = gelu_erf(round16<DT>(v3));
      }
      *reinterpret_cast<uint2*>(p.C + static_cast<long long>(row) * p.ldc + c) =
          make_uint2(pack2<DT>(v0, v1), pack2<DT>(v2, v3));
    }
  }
}

// Split-K residual projection closed by the LayerNorm of its result, one
// 128-thread block per row (4 consecutive columns per thread and chunk, NC4
// chunks, so that a few-row input still spreads over many SMs):
//   x_out  = mask_x(x_in + mask_delta(sum of the partials + bias))   (EPI 2;
//            EPI 4 with the half-precision model's roundings to DT)
//   normed = mask_out(LayerNorm(x_out) * w + b)
// The partials are summed in split order, as splitk_reduce_kernel does, so
// x_out is bit-identical to the unfused reduce; the moments are two-pass
// (mean, then the centred sum of squares) as in the LayerNorm kernels. For
// few-row inputs every kernel is latency-bound, and this saves the separate
// LayerNorm launch of each residual site.
constexpr int kRlnThreads = 128;

__device__ __forceinline__ float block_sum_rln(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // red is reused by consecutive reductions
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

template <int NC4, int EPI, int DT>
__global__ void __launch_bounds__(kRlnThreads) splitk_reduce_ln_kernel(const GemmArgs p, const LnFuse ln) {
  __shared__ float red[kRlnThreads / 32];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const int N = p.N;
  const long long plane = static_cast<long long>(p.M) * N;
  const bool valid = p.valid == nullptr || p.valid[row] != 0;
  float v[NC4][4];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NC4; ++i) {
    const int col = 4 * (static_cast<int>(threadIdx.x) + kRlnThreads * i);
    if (col < N) {
      const float* src = p.ws + row * N + col;
      float4 a = *reinterpret_cast<const float4*>(src);
#pragma unroll 4
      for (int sp = 1; sp < p.splits; ++sp) {
        const float4 b = *reinterpret_cast<const float4*>(src + sp * plane);
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
      }
      const float4 q = __ldg(reinterpret_cast<const float4*>(p.bias + col));
      const float d[4] = {a.x + q.x, a.y + q.y, a.z + q.z, a.w + q.w};
      const long long off = row * p.ldx + col;
      float x[4];
      if constexpr (EPI == 4) {
        const uint2 h = *reinterpret_cast<const uint2*>(p.x16_in + off);
        const float2 f0 = unpack2<DT>(h.x), f1 = unpack2<DT>(h.y);
        x[0] = f0.x; x[1] = f0.y; x[2] = f1.x; x[3] = f1.y;
      } else {
        const float4 x0 = *reinterpret_cast<const float4*>(p.x_in + off);
        x[0] = x0.x; x[1] = x0.y; x[2] = x0.z; x[3] = x0.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float dj = EPI == 4 ? round16<DT>(d[j]) : d[j];
        if (p.mask_mode == 1 && !valid) dj = 0.f;
        float y = x[j] + dj;
        if constexpr (EPI == 4) y = round16<DT>(y);
        if (p.mask_mode == 2 && !valid) y = 0.f;
        v[i][j] = y;
        sum += y;
      }
      if constexpr (EPI == 4) {
        *reinterpret_cast<uint2*>(p.x16_out + off) = make_uint2(pack2<DT>(v[i][0], v[i][1]), pack2<DT>(v[i][2], v[i][3]));
      } else {
        *reinterpret_cast<float4*>(p.x_out + off) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
      }
    }
  }
  const float mean = block_sum_rln(sum, red) / static_cast<float>(N);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NC4; ++i) {
    if (4 * (static_cast<int>(threadIdx.x) + kRlnThreads * i) < N) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float dv = v[i][j] - mean;
        sq += dv * dv;
      }
    }
  }
  const float rstd = rsqrtf(block_sum_rln(sq, red) / static_cast<float>(N) + ln.eps);
  const bool zero_out = (ln.flags & TF_LN_MASK_OUT) && !valid;
#pragma unroll
  for (int i = 0; i < NC4; ++i) {
    const int col = 4 * (static_cast<int>(threadIdx.x) + kRlnThreads * i);
    if (col < N) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(ln.w + col));
      const float4 bv = __ldg(reinterpret_cast<const float4*>(ln.b + col));
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, ba[4] = {bv.x, bv.y, bv.z, bv.w};
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = zero_out ? 0.f : (v[i][j] - mean) * rstd * wa[j] + ba[j];
      const long long off = row * N + col;
      if (ln.flags & TF_LN_OUT_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(ln.normed) + off) = make_float4(y[0], y[1], y[2], y[3]);
      } else {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(ln.normed) + off) =
            make_uint2(pack2<DT>(y[0], y[1]), pack2<DT>(y[2], y[3]));
      }
    }
  }
}

// Split count and workspace bytes of a split-K call. splits <= 0: automatic,
// about one work unit per two SMs and at least two k-blocks (128 of K) per
// unit (measured on the small model configs: more splits only add partials
// for the reduce kernel to read).
static void splitk_plan(long long M, long long N, long long K, int splits_req, int sms, int& splits, int& kps) {
  const long long tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + 63) / 64);
  const int k_blocks = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  long long sp = splits_req;
  if (sp <= 0) {
    sp = tiles * 2 >= sms ? 1 : sms / (2 * tiles);
    if (sp > k_blocks / 2) sp = k_blocks / 2;
  }
  if (sp > k_blocks) sp = k_blocks;
  if (sp > kMaxSplits) sp = kMaxSplits;
  if (sp < 1) sp = 1;
  kps = static_cast<int>((k_blocks + sp - 1) / sp);
  splits = (k_blocks + kps - 1) / kps;  // no empty split
}

long long gemm_splitk_workspace_bytes(long long M, long long N, long long K, int splits_req) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int splits, kps;
  splitk_plan(M, N, K, splits_req, device_sm_count(), splits, kps);
  return static_cast<long long>(splits) * M * N * 4;
}

int gemm_splitk_f16(const GemmCall& g, int splits_req, float* ws, long long ws_bytes, cudaStream_t stream,
                    const LnFuse* ln) {
  const long long M = g.M, N = g.N, K = g.K;
  if (M <= 0 || N <= 0 || K <= 0) return set_error(TF_ERR_SHAPE, "gemm_splitk: empty shape M=%lld N=%lld K=%lld", M, N, K);
  if (M > (1ll << 31) - 1 || N > 65535ll * 64 || K > (1 << 24)) return set_error(TF_ERR_SHAPE, "gemm_splitk: shape out of range");
  if (N % 32 != 0) return set_error(TF_ERR_SHAPE, "gemm_splitk: N=%lld must be a multiple of 32", N);
  if (g.a_repeat != 1) return set_error(TF_ERR_SHAPE, "gemm_splitk: split weights are not supported");
  if (g.epilogue < 0 || g.epilogue > 5 || g.epilogue == 3)
    return set_error(TF_ERR_SHAPE, "gemm_splitk: epilogue %d", g.epilogue);
  if (g.dtype != kDtF16 && g.dtype != kDtBF16) return set_error(TF_ERR_SHAPE, "gemm_splitk: operand type %d", g.dtype);
  if (K % 8 != 0 || g.lda % 8 != 0 || g.ldw % 8 != 0)
    return set_error(TF_ERR_ALIGN, "gemm_splitk: K and leading dimensions must be multiples of 8 elements");
  if (g.lda < K || g.ldw < K) return set_error(TF_ERR_SHAPE, "gemm_splitk: leading dimension smaller than row");
  if (!aligned16(g.A) || !aligned16(g.W) || !aligned16(g.bias) || g.A == nullptr || g.W == nullptr ||
      g.bias == nullptr)
    return set_error(TF_ERR_ALIGN, "gemm_splitk: A, W and bias must be non-null and 16-byte aligned");
  if (g.epilogue == 2 || g.epilogue == 4) {
    const int mult = g.epilogue == 2 ? 4 : 8;
    if (g.x_in == nullptr || g.x_out == nullptr || !aligned16(g.x_in) || !aligned16(g.x_out) || g.ldx % mult != 0 ||
        g.ldx < N)
      return set_error(TF_ERR_ALIGN,
                       "gemm_splitk: x_in/x_out must be 16-byte aligned with a pitch >= N, multiple of %d", mult);
    if (g.mask_mode < 0 || g.mask_mode > 2) return set_error(TF_ERR_SHAPE, "gemm_splitk: mask mode %d", g.mask_mode);
    if (g.mask_mode != 0 && g.valid == nullptr) return set_error(TF_ERR_SHAPE, "gemm_splitk: mask without valid rows");
  } else if (g.C == nullptr || !aligned16(g.C) || g.ldc % 8 != 0 || g.ldc < N) {
    return set_error(TF_ERR_ALIGN, "gemm_splitk: C must be 16-byte aligned with a pitch >= N, multiple of 8");
  }
  if (ln != nullptr) {
    if (g.epilogue != 2 && g.epilogue != 4)
      return set_error(TF_ERR_SHAPE, "gemm_splitk: the fused LayerNorm follows a residual epilogue only");
    if (N > 4096) return set_error(TF_ERR_SHAPE, "gemm_splitk: fused LayerNorm rows of %lld > 4096", N);
    if (ln->w == nullptr || ln->b == nullptr || ln->normed == nullptr || !aligned16(ln->w) || !aligned16(ln->b) ||
        !aligned16(ln->normed))
      return set_error(TF_ERR_ALIGN, "gemm_splitk: LayerNorm weight, bias and output must be non-null, 16-byte aligned");
    if (ln->flags & ~(TF_LN_MASK_OUT | TF_LN_OUT_F32))
      return set_error(TF_ERR_SHAPE, "gemm_splitk: LayerNorm flags %d (TF_LN_MASK_OUT, TF_LN_OUT_F32)", ln->flags);
    if ((ln->flags & TF_LN_MASK_OUT) && g.valid == nullptr)
      return set_error(TF_ERR_SHAPE, "gemm_splitk: TF_LN_MASK_OUT without valid rows");
  }
  const int sms = device_sm_count();
  int splits, kps;
  splitk_plan(M, N, K, splits_req, sms, splits, kps);
  const long long need = static_cast<long long>(splits) * M * N * 4;
  if (ws == nullptr || !aligned16(ws) || ws_bytes < need)
    return set_error(TF_ERR_SHAPE, "gemm_splitk: workspace of %lld bytes (16-byte aligned) needed, %lld given", need,
                     ws_bytes);

  CUtensorMap ta, tb;
  int rc = make_tmap_2d_f16(&ta, g.A, K, M, g.lda, kGemmBK, 128);
  if (rc) return rc;
  rc = make_tmap_2d_f16(&tb, g.W, K, N, g.ldw, kGemmBK, 64);
  if (rc) return rc;

  GemmArgs args = make_args(g);
  args.a_repeat = 1;
  args.m_tiles = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  args.n_tiles = static_cast<int>((N + 63) / 64);
  args.status = device_status_ptr();
  if (args.status == nullptr) return last_error_code();
  args.splits = splits;
  args.kb_per_split = kps;
  args.ws = ws;
  const long long units = static_cast<long long>(args.m_tiles) * args.n_tiles * splits;
  const int grid = static_cast<int>(units < sms ? units : sms);
  rc = g.dtype == kDtBF16 ? launch_gemm_cfg<64, 8, 3, kDtBF16>(ta, tb, args, grid, stream)
                          : launch_gemm_cfg<64, 8, 3, kDtF16>(ta, tb, args, grid, stream);
  if (rc) return rc;

  if (ln != nullptr) {
    // one block per row
    const dim3 lgrid(static_cast<unsigned>(M));
    const int n4 = static_cast<int>((N / 4 + kRlnThreads - 1) / kRlnThreads);
    const int nc = n4 <= 1 ? 1 : n4 <= 2 ? 2 : n4 <= 4 ? 4 : 8;
    cudaError_t e = cudaSuccess;
#define TFB_RLN(C, E, D) e = launch_k(splitk_reduce_ln_kernel<C, E, D>, lgrid, dim3(kRlnThreads), 0, stream, args, *ln)
#define TFB_RLN_NCH(E, D)                 \
  switch (nc) {                           \
    case 1: TFB_RLN(1, E, D); break;      \
    case 2: TFB_RLN(2, E, D); break;      \
    case 4: TFB_RLN(4, E, D); break;      \
    default: TFB_RLN(8, E, D); break;     \
  }
    if (g.epilogue == 2) {
      TFB_RLN_NCH(2, kDtF16)
    } else if (g.dtype == kDtBF16) {
      TFB_RLN_NCH(4, kDtBF16)
    } else {
      TFB_RLN_NCH(4, kDtF16)
    }
#undef TFB_RLN_NCH
#undef TFB_RLN
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "gemm_splitk reduce+LayerNorm launch: %s", cudaGetErrorString(e));
    return TF_OK;
  }
  const long long nq = M * (N / 4);
  long long blocks = (nq + 255) / 256;
  if (blocks > 8ll * sms) blocks = 8ll * sms;
  cudaError_t e;
  const dim3 rgrid(static_cast<unsigned>(blocks));
#define TFB_REDUCE_CASE(E, D) \
  case E * 2 + D: e = launch_k(splitk_reduce_kernel<E, D>, rgrid, dim3(256), 0, stream, args); break;
  switch (g.epilogue * 2 + g.dtype) {
    TFB_REDUCE_CASE(0, 0)
    TFB_REDUCE_CASE(1, 0)
    TFB_REDUCE_CASE(2, 0)
    TFB_REDUCE_CASE(4, 0)
    TFB_REDUCE_CASE(5, 0)
    TFB_REDUCE_CASE(0, 1)
    TFB_REDUCE_CASE(1, 1)
    TFB_REDUCE_CASE(2, 1)
    TFB_REDUCE_CASE(4, 1)
    default: e = launch_k(splitk_reduce_kernel<5, 1>, rgrid, dim3(256), 0, stream, args); break;
  }
#undef TFB_REDUCE_CASE
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "gemm_splitk reduce launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

// ---------------------------------------------------------------------------
// Split-K with library-owned scratch: the fp32 partials go to a fixed device
// array of this library instead of a caller workspace, for callers that
// cannot allocate device memory (see tf_gemm_splitk_static).
// ---------------------------------------------------------------------------
constexpr long long kStaticScratchBytes = 4ll << 20;  // 4 MiB of fp32 partial sums
static __device__ __align__(256) float g_splitk_scratch[kStaticScratchBytes / 4];

int gemm_splitk_static_f16(const GemmCall& g, int splits, cudaStream_t stream) {
  static std::mutex mu;
  static float* ptrs[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TF_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(TF_ERR_DEVICE, "device ordinal %d out of range", dev);
  float* scratch;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[dev] == nullptr) {
      // once per device, with that device current: the address of this
      // device's copy of the array (no allocation; the array is part of the
      // library's device image)
      void* a = nullptr;
      e = cudaGetSymbolAddress(&a, g_splitk_scratch);
      if (e != cudaSuccess) return set_error(TF_ERR_DEVICE, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
      ptrs[dev] = static_cast<float*>(a);
    }
    scratch = ptrs[dev];
  }
  const long long need = gemm_splitk_workspace_bytes(g.M, g.N, g.K, splits);
  if (need > kStaticScratchBytes)
    return set_error(TF_ERR_SHAPE, "gemm_splitk_static: %lld bytes of partial sums exceed the %lld-byte scratch", need,
                     kStaticScratchBytes);
  // every partial element a call reads is written by the same call first, so
  // the scratch needs no clearing between calls
  return gemm_splitk_f16(g, splits, scratch, kStaticScratchBytes, stream);
}

}  // namespace tfb
