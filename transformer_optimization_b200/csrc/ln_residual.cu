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
// Half-precision models (XT = kLnF16 / kLnBF16): x, delta and x_out are in the
// model's type T and the sum is rounded to T before the statistics, as the
// eager model stores `x = x + delta` in T before nn.LayerNorm reads it
// (torch_transformer_benchmark.py:218-222); normed is T (or fp32).
//
// HBM-bound: bytes per row = D*(4 read x + 2 read delta + 4 write x + 2 write
// normed). Two kernels:
//  * ln_stream_kernel (D <= 2048): one persistent CTA per SM streams groups of
//    8 rows through a ring of shared-memory stages filled by the bulk-copy
//    engine (cp.async.bulk, one copy for the 8 x rows and one for the 8 delta
//    rows of a group), so ~100-200 KB per SM are in flight independent of
//    registers; two or three teams of 8 consumer warps take successive
//    groups, one row per warp, and store the results straight to HBM.
//  * ln_residual_kernel (any D up to 4096): one warp per row with the row in
//    registers, grid-stride over rows.
//
// Ready mode (ln_stream_kernel, no delta): the rows come from a residual GEMM
// that is still running (tf_gemm_residual_ready). Its epilogue counts the
// stored columns of every 8-row group; this kernel does not wait for the GEMM
// grid to finish (no griddepcontrol.wait) but, per group, for the group's
// count to reach D, then copies it and zeroes the count for the next site.
// The groups are handed out in ascending order from a ticket counter (two
// ints after the group counts), one at a time per CTA and only after the
// CTA's previous group was complete: the CTAs that start first (on the SMs
// the GEMM's last, partial wave leaves idle) take the rows the GEMM finished
// first, and once the GEMM ends every CTA shares what is left. The last CTA
// to run out of tickets zeroes the ticket counters.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kLnRowsPerBlock = 8;

// Element type of the residual stream x (and of delta and x_out): the fp32
// model keeps x in fp32 with an fp16 delta; the half-precision models keep
// all three in their own 16-bit type.
constexpr int kLnF32 = 0;
constexpr int kLnF16 = 1;
constexpr int kLnBF16 = 2;
template <int XT>
constexpr int kLnDt = XT == kLnBF16 ? kDtBF16 : kDtF16;  // type of delta and of a 16-bit normed

// Four consecutive elements of a 16-bit row of type DT, widened.
template <int DT>
__device__ __forceinline__ void widen4(uint2 q, float (&v)[4]) {
  const float2 a = unpack2<DT>(q.x), b = unpack2<DT>(q.y);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

template <int NCH, int XT>  // 8-element chunks per lane (row width up to 256*NCH); x's type
__global__ void __launch_bounds__(256) ln_residual_kernel(const void* __restrict__ x,
                                                          const uint16_t* __restrict__ delta,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ b, float eps,
                                                          const uint8_t* __restrict__ valid, long long M, int D,
                                                          int flags, void* __restrict__ x_out,
                                                          void* __restrict__ normed) {
  constexpr int DT = kLnDt<XT>;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long warps_total = static_cast<long long>(gridDim.x) * kLnRowsPerBlock;
  for (long long row = static_cast<long long>(blockIdx.x) * kLnRowsPerBlock + (threadIdx.x >> 5); row < M;
       row += warps_total) {
  const int nchunk = D >> 3;
  bool row_valid = true;
  if (valid != nullptr) row_valid = valid[row] != 0;

  float v[NCH][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nchunk) {
      if constexpr (XT == kLnF32) {
        const float* xr = static_cast<const float*>(x) + row * D;
        const float4 a0 = __ldcs(reinterpret_cast<const float4*>(xr) + 2 * c);
        const float4 a1 = __ldcs(reinterpret_cast<const float4*>(xr) + 2 * c + 1);
        v[i][0] = a0.x; v[i][1] = a0.y; v[i][2] = a0.z; v[i][3] = a0.w;
        v[i][4] = a1.x; v[i][5] = a1.y; v[i][6] = a1.z; v[i][7] = a1.w;
      } else {
        const uint4 q = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + row * D) + c);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack2<DT>(qw[j]);
          v[i][2 * j] = f.x;
          v[i][2 * j + 1] = f.y;
        }
      }
      if (delta != nullptr) {
        const uint4 dq = __ldcs(reinterpret_cast<const uint4*>(delta + row * D) + c);
        const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
        const bool keep = !(flags & TF_LN_MASK_DELTA) || row_valid;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack2<DT>(dw[j]);
          v[i][2 * j] += keep ? f.x : 0.f;
          v[i][2 * j + 1] += keep ? f.y : 0.f;
        }
        if constexpr (XT != kLnF32) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = round16<DT>(v[i][j]);
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
        if constexpr (XT == kLnF32) {
          float4* xo = reinterpret_cast<float4*>(static_cast<float*>(x_out) + row * D) + 2 * c;
          __stcs(xo, make_float4(v[i][0], v[i][1], v[i][2], v[i][3]));
          __stcs(xo + 1, make_float4(v[i][4], v[i][5], v[i][6], v[i][7]));
        } else {
          __stcs(reinterpret_cast<uint4*>(static_cast<uint16_t*>(x_out) + row * D) + c,
                 make_uint4(pack2<DT>(v[i][0], v[i][1]), pack2<DT>(v[i][2], v[i][3]), pack2<DT>(v[i][4], v[i][5]),
                            pack2<DT>(v[i][6], v[i][7])));
        }
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
        q.x = pack2<DT>(y[0], y[1]);
        q.y = pack2<DT>(y[2], y[3]);
        q.z = pack2<DT>(y[4], y[5]);
        q.w = pack2<DT>(y[6], y[7]);
        reinterpret_cast<uint4*>(static_cast<uint16_t*>(normed) + row * D)[c] = q;
      }
    }
  }
  }  // row loop
}


// ---------------------------------------------------------------------------
// Streaming variant: bulk-copy ring of 8-row groups
// ---------------------------------------------------------------------------
constexpr int kLnsRows = 8;        // rows per group (one consumer warp each)
constexpr int kLnsMaxStages = 8;
// TEAMS consumer teams of 8 warps work on successive groups, + 1 producer warp
__host__ __device__ constexpr int lns_threads(int teams) { return 32 * (kLnsRows * teams + 1); }
constexpr int kLnsSmemBudget = 196608;

struct LnsParams {
  const void* x;
  const uint16_t* delta;
  const float* w;
  const float* b;
  const uint8_t* valid;
  void* x_out;
  void* normed;
  long long M;
  int D, flags, stages;
  float eps;
  int* status;
  int* ready;  // ready mode: per-8-row-group stored-column counts, else null
};

// Stage ownership: group number `it` (this CTA's it-th group) goes to stage
// it % stages and to team it % TEAMS. The host makes stages a multiple of
// TEAMS, so every stage is only ever used by one team, whose waits on it come
// in phase order: an mbarrier waiter that could fall two phases behind would
// see the parity of an older phase and read a stage that is being refilled.
template <int NV, int TEAMS, int XT>  // NV: 4-element vectors per lane (row width up to 128*NV); x's type
__global__ void __launch_bounds__(lns_threads(TEAMS), 1) ln_stream_kernel(const LnsParams p) {
  constexpr int DT = kLnDt<XT>;
  constexpr int XS = XT == kLnF32 ? 4 : 2;  // bytes per x element
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int D = p.D;
  const bool has_delta = p.delta != nullptr;
  const uint32_t x_bytes = static_cast<uint32_t>(kLnsRows) * D * XS;
  const uint32_t stage_bytes = x_bytes + (has_delta ? static_cast<uint32_t>(kLnsRows) * D * 2 : 0u);
  // LayerNorm weight and bias staged once per CTA (read by every row)
  float* w_s = reinterpret_cast<float*>(smem + p.stages * stage_bytes);
  float* b_s = w_s + D;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_s + D);
  uint64_t* empty = full + kLnsMaxStages;
  int* stage_group = reinterpret_cast<int*>(empty + kLnsMaxStages);  // ready mode: group in a stage, -1 = none left
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long groups = (p.M + kLnsRows - 1) / kLnsRows;
  if (p.stages % TEAMS != 0 || p.stages > kLnsMaxStages) {  // host invariant; refuse rather than race
    if (threadIdx.x == 0) record_error(p.status, kDevTimeoutProducer);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kLnsRows);
    }
    fence_mbar_init();
  }
  // ready mode reads only rows whose counts are complete and writes only
  // `normed`, which no kernel still running reads
  if (p.ready == nullptr) pdl_wait();
  pdl_trigger();
  // this CTA's groups: strided over the grid (its it-th group is
  // blockIdx.x + it * gridDim.x), or (ready mode) drawn from the ticket counter
  const bool dynamic = p.ready != nullptr;
  const long long n_mine = dynamic ? 0x7fffffff : (groups - blockIdx.x + gridDim.x - 1) / gridDim.x;
  for (int i = threadIdx.x; i < (D >> 2); i += blockDim.x) {
    reinterpret_cast<float4*>(w_s)[i] = __ldg(reinterpret_cast<const float4*>(p.w) + i);
    reinterpret_cast<float4*>(b_s)[i] = __ldg(reinterpret_cast<const float4*>(p.b) + i);
  }
  __syncthreads();

  if (warp == kLnsRows * TEAMS) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int* ticket = dynamic ? p.ready + groups : nullptr;  // next group to hand out
      int* done = ticket + 1;                              // CTAs out of tickets
      bool ok = true;
      int it = 0;
      for (; it < n_mine; ++it) {
        const int s = it % p.stages;
        if (!(ok = mbar_wait(&empty[s], ((it / p.stages) & 1) ^ 1, p.status, kDevTimeoutProducer))) break;
        long long g = blockIdx.x + static_cast<long long>(it) * gridDim.x;
        if (dynamic) {
          g = atomicAdd(ticket, 1);
          if (g >= groups) break;  // stage s (already free) takes the first stop below
          stage_group[s] = static_cast<int>(g);
          if (!(ok = wait_ready(p.ready + g, D, p.status))) break;
          fence_proxy_async_global();
          p.ready[g] = 0;  // consumed; the next site's GEMM starts after this grid ends
        }
        const long long r0 = g * kLnsRows;
        const int nrows = static_cast<int>(p.M - r0 < kLnsRows ? p.M - r0 : kLnsRows);
        uint8_t* st = smem + s * stage_bytes;
        const uint32_t xb = static_cast<uint32_t>(nrows) * D * XS;
        const uint32_t db = has_delta ? static_cast<uint32_t>(nrows) * D * 2 : 0u;
        mbar_arrive_expect_tx(&full[s], xb + db);
        bulk_load_1d(st, static_cast<const uint8_t*>(p.x) + r0 * D * XS, xb, &full[s]);
        if (has_delta) bulk_load_1d(st + x_bytes, p.delta + r0 * D, db, &full[s]);
      }
      if (dynamic && ok) {
        // one stop per team: the stages of this CTA's next TEAMS groups
        for (int k = 0; k < TEAMS && ok; ++k, ++it) {
          const int s = it % p.stages;
          if (k > 0 && !(ok = mbar_wait(&empty[s], ((it / p.stages) & 1) ^ 1, p.status, kDevTimeoutProducer)))
            break;
          stage_group[s] = -1;
          mbar_arrive(&full[s]);
        }
        // no CTA draws a ticket after the last one has run out: reset both
        if (atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1) {
          *ticket = 0;
          *done = 0;
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  // team k = warp / 8 takes this CTA's groups k, k+TEAMS, ...; warp w of the
  // team takes row w % 8 of each
  const int nv = D >> 2;  // 4-element vectors per row
  const int team = warp / kLnsRows, wr = warp % kLnsRows;
  for (int it = team; it < n_mine; it += TEAMS) {
    const int s = it % p.stages;
    long long g = blockIdx.x + static_cast<long long>(it) * gridDim.x;
    long long row = g * kLnsRows + wr;
    bool row_valid = true;
    if (!dynamic && p.valid != nullptr && row < p.M) row_valid = p.valid[row] != 0;  // ahead of the wait
    // ready mode: a stage can stay empty for as long as the producer's count
    // wait (bounded by kWaitLimitNs itself), so the consumers wait twice that
    // and leave as soon as the producer records why it gave up
    if (!mbar_wait_ns(&full[s], (it / p.stages) & 1, p.status, kDevTimeoutEpilogue,
                      dynamic ? 2 * kWaitLimitNs : kWaitLimitNs))
      break;
    if (dynamic) {
      g = stage_group[s];
      if (g < 0) break;  // no group left for this team
      row = g * kLnsRows + wr;
      if (p.valid != nullptr && row < p.M) row_valid = p.valid[row] != 0;
    }
    const bool have = row < p.M;
    if (have) {
      const uint8_t* xrow = smem + s * stage_bytes + static_cast<long long>(wr) * D * XS;
      const uint2* ds = reinterpret_cast<const uint2*>(smem + s * stage_bytes + x_bytes) + static_cast<long long>(wr) * nv;
      const bool keep = !(p.flags & TF_LN_MASK_DELTA) || row_valid;
      const bool zero_x = (p.flags & TF_LN_MASK_X) && !row_valid;
      float v[NV][4];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = lane + 32 * i;
        if (c < nv) {
          if constexpr (XT == kLnF32) {
            const float4 a = reinterpret_cast<const float4*>(xrow)[c];
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
          } else {
            widen4<DT>(reinterpret_cast<const uint2*>(xrow)[c], v[i]);
          }
          if (has_delta && keep) {
            float d[4];
            widen4<DT>(ds[c], d);
            v[i][0] += d[0]; v[i][1] += d[1]; v[i][2] += d[2]; v[i][3] += d[3];
            if constexpr (XT != kLnF32) {
#pragma unroll
              for (int j = 0; j < 4; ++j) v[i][j] = round16<DT>(v[i][j]);
            }
          }
          if (zero_x) v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.f;
          sum += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // the row is in registers
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float mean = sum / static_cast<float>(D);
      float sq = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (lane + 32 * i < nv) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float d = v[i][j] - mean;
            sq += d * d;
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      const float rstd = rsqrtf(sq / static_cast<float>(D) + p.eps);
      const bool zero_out = (p.flags & TF_LN_MASK_OUT) && !row_valid;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = lane + 32 * i;
        if (c < nv) {
          if (p.flags & TF_LN_WRITE_X) {
            if constexpr (XT == kLnF32) {
              __stcs(reinterpret_cast<float4*>(static_cast<float*>(p.x_out) + row * D) + c,
                     make_float4(v[i][0], v[i][1], v[i][2], v[i][3]));
            } else {
              __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.x_out) + row * D) + c,
                     make_uint2(pack2<DT>(v[i][0], v[i][1]), pack2<DT>(v[i][2], v[i][3])));
            }
          }
          const float4 wv = reinterpret_cast<const float4*>(w_s)[c];
          const float4 bv = reinterpret_cast<const float4*>(b_s)[c];
          float y0 = (v[i][0] - mean) * rstd * wv.x + bv.x;
          float y1 = (v[i][1] - mean) * rstd * wv.y + bv.y;
          float y2 = (v[i][2] - mean) * rstd * wv.z + bv.z;
          float y3 = (v[i][3] - mean) * rstd * wv.w + bv.w;
          if (zero_out) y0 = y1 = y2 = y3 = 0.f;
          if (p.flags & TF_LN_OUT_F32) {
            __stcs(reinterpret_cast<float4*>(static_cast<float*>(p.normed) + row * D) + c, make_float4(y0, y1, y2, y3));
          } else {
            __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.normed) + row * D) + c,
                   make_uint2(pack2<DT>(y0, y1), pack2<DT>(y2, y3)));
          }
        }
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
}

template <int XT>
static int ln_launch(const void* x, const void* delta, const float* w, const float* b, float eps,
                     const uint8_t* valid, long long M, int D, int flags, void* x_out, void* normed,
                     cudaStream_t stream, int* ready = nullptr) {
  constexpr int XS = XT == kLnF32 ? 4 : 2;
  if (ready != nullptr && D > 2048) return set_error(TF_ERR_SHAPE, "ln_ready: D=%d above 2048", D);
  if (D <= 2048) {
    LnsParams lp;
    lp.x = x;
    lp.delta = static_cast<const uint16_t*>(delta);
    lp.w = w;
    lp.b = b;
    lp.valid = valid;
    lp.x_out = x_out;
    lp.normed = normed;
    lp.M = M;
    lp.D = D;
    lp.flags = flags;
    lp.eps = eps;
    lp.status = device_status_ptr();
    if (lp.status == nullptr) return last_error_code();
    lp.ready = ready;
    const int stage_bytes = kLnsRows * D * (XS + (delta != nullptr ? 2 : 0));
    // teams and stages (a multiple of the team count, see the kernel's
    // stage-ownership note), best measured at the c3/c4 shapes: three teams
    // with six stages (D <= 1024 without delta), two with four (D = 1024 with
    // delta), three with three (D = 2048), two with two (D = 2048 with delta)
    int fit = kLnsSmemBudget / stage_bytes;
    if (fit > kLnsMaxStages) fit = kLnsMaxStages;
    const int teams = (fit >= 6 || fit == 3) ? 3 : 2;
    const int stages = (fit / teams) * teams;
    if (stages < teams) return set_error(TF_ERR_SHAPE, "ln_residual: D=%d too wide for the streaming kernel", D);
    lp.stages = stages;
    const int smem = stages * stage_bytes + 8 * D + 2 * kLnsMaxStages * 8 + kLnsMaxStages * 4 + 128;
    const long long groups = (M + kLnsRows - 1) / kLnsRows;
    const long long grid = groups < device_sm_count() ? groups : device_sm_count();
    const int nv = (D / 4 + 31) / 32;
    int dev = 0;
    cudaGetDevice(&dev);
#define TFB_LNS_CASE(N, T)                                                                          \
  {                                                                                                 \
    static bool attr_done[64] = {};                                                                 \
    if (!attr_done[dev & 63]) {                                                                     \
      cudaError_t ea = cudaFuncSetAttribute(ln_stream_kernel<N, T, XT>,                             \
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,            \
                                            kLnsSmemBudget + 8 * 2048 + 2 * kLnsMaxStages * 8 + kLnsMaxStages * 4 + 128); \
      if (ea != cudaSuccess)                                                                        \
        return set_error(TF_ERR_LAUNCH, "cudaFuncSetAttribute(ln): %s", cudaGetErrorString(ea));    \
      attr_done[dev & 63] = true;                                                                   \
    }                                                                                               \
    launch_k(ln_stream_kernel<N, T, XT>, dim3(static_cast<unsigned>(grid)), dim3(lns_threads(T)), smem, stream, \
             lp);                                                                                   \
  }                                                                                                 \
  break;
    const int nvc = nv <= 2 ? 2 : nv <= 4 ? 4 : nv <= 8 ? 8 : 16;
    switch (nvc * 10 + teams) {
      case 22: TFB_LNS_CASE(2, 2)
      case 23: TFB_LNS_CASE(2, 3)
      case 42: TFB_LNS_CASE(4, 2)
      case 43: TFB_LNS_CASE(4, 3)
      case 82: TFB_LNS_CASE(8, 2)
      case 83: TFB_LNS_CASE(8, 3)
      case 162: TFB_LNS_CASE(16, 2)
      default: TFB_LNS_CASE(16, 3)
    }
#undef TFB_LNS_CASE
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "ln_residual launch: %s", cudaGetErrorString(e));
    return TF_OK;
  }
  // grid-stride over rows with the device filled exactly (resident blocks
  // per SM from the occupancy of this instantiation)
  const int nch = (D / 8 + 31) / 32;
  const uint16_t* dh = static_cast<const uint16_t*>(delta);
  const long long need = (M + kLnRowsPerBlock - 1) / kLnRowsPerBlock;
#define TFB_LN_CASE(N)                                                                                        \
  {                                                                                                           \
    int per_sm = 1;                                                                                           \
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ln_residual_kernel<N, XT>, 256, 0);                \
    long long blocks = static_cast<long long>(device_sm_count()) * (per_sm > 0 ? per_sm : 1);                 \
    if (blocks > need) blocks = need;                                                                         \
    launch_k(ln_residual_kernel<N, XT>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, x, dh, w, b, \
             eps, valid, M, D, flags, x_out, normed);                                                        \
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

int ln_residual(const void* x, const void* delta, const float* w, const float* b, float eps,
                const uint8_t* valid, long long M, int D, int flags, void* x_out, void* normed,
                cudaStream_t stream) {
  if (M <= 0) return TF_OK;  // nothing to do
  if (D <= 0 || D % 8 != 0 || D > 4096)
    return set_error(TF_ERR_SHAPE, "ln_residual: D=%d must be a positive multiple of 8, <= 4096", D);
  if ((flags & TF_LN_X_F16) && (flags & TF_LN_X_BF16))
    return set_error(TF_ERR_SHAPE, "ln_residual: TF_LN_X_F16 and TF_LN_X_BF16 together");
  if (!aligned16(x) || !aligned16(delta) || !aligned16(w) || !aligned16(b) || !aligned16(x_out) ||
      !aligned16(normed))
    return set_error(TF_ERR_ALIGN, "ln_residual: pointers must be 16-byte aligned");
  if (x == nullptr || w == nullptr || b == nullptr || normed == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_residual: x, w, b and normed are required");
  if ((flags & TF_LN_WRITE_X) && x_out == nullptr) return set_error(TF_ERR_SHAPE, "ln_residual: WRITE_X without x_out");
  if ((flags & (TF_LN_MASK_DELTA | TF_LN_MASK_X | TF_LN_MASK_OUT)) && valid == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_residual: mask flag without a valid-token mask");
  if (!(flags & (TF_LN_MASK_DELTA | TF_LN_MASK_X | TF_LN_MASK_OUT))) valid = nullptr;
  if (flags & TF_LN_X_BF16)
    return ln_launch<kLnBF16>(x, delta, w, b, eps, valid, M, D, flags, x_out, normed, stream);
  if (flags & TF_LN_X_F16)
    return ln_launch<kLnF16>(x, delta, w, b, eps, valid, M, D, flags, x_out, normed, stream);
  return ln_launch<kLnF32>(x, delta, w, b, eps, valid, M, D, flags, x_out, normed, stream);
}

int ln_ready(const void* x, const float* w, const float* b, float eps, const uint8_t* valid, long long M, int D,
             int flags, void* normed, int* ready, cudaStream_t stream) {
  if (M <= 0) return TF_OK;
  if (D <= 0 || D % 8 != 0 || D > 2048)
    return set_error(TF_ERR_SHAPE, "ln_ready: D=%d must be a positive multiple of 8, <= 2048", D);
  if (flags & ~(TF_LN_MASK_OUT | TF_LN_OUT_F32 | TF_LN_X_F16 | TF_LN_X_BF16))
    return set_error(TF_ERR_SHAPE, "ln_ready: flags %d (only MASK_OUT, OUT_F32, X_F16, X_BF16)", flags);
  if ((flags & TF_LN_X_F16) && (flags & TF_LN_X_BF16))
    return set_error(TF_ERR_SHAPE, "ln_ready: TF_LN_X_F16 and TF_LN_X_BF16 together");
  if (x == nullptr || w == nullptr || b == nullptr || normed == nullptr || ready == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_ready: x, w, b, normed and ready are required");
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(normed) ||
      reinterpret_cast<uintptr_t>(ready) % 4 != 0)
    return set_error(TF_ERR_ALIGN, "ln_ready: x, w, b, normed 16-byte aligned, ready 4-byte aligned");
  if ((flags & TF_LN_MASK_OUT) && valid == nullptr)
    return set_error(TF_ERR_SHAPE, "ln_ready: TF_LN_MASK_OUT without a valid-token mask");
  if (!(flags & TF_LN_MASK_OUT)) valid = nullptr;
  if (flags & TF_LN_X_BF16)
    return ln_launch<kLnBF16>(x, nullptr, w, b, eps, valid, M, D, flags, nullptr, normed, stream, ready);
  if (flags & TF_LN_X_F16)
    return ln_launch<kLnF16>(x, nullptr, w, b, eps, valid, M, D, flags, nullptr, normed, stream, ready);
  return ln_launch<kLnF32>(x, nullptr, w, b, eps, valid, M, D, flags, nullptr, normed, stream, ready);
}

}  // namespace tfb
