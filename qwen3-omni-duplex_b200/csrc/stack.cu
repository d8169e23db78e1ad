// Persistent clock-path kernel: every int4 linear of L Thinker layers for T <= 8
// decode tokens in ONE launch (one CTA per SM, 16 consumer warps + 1 producer warp).
//
// Per layer the consumers run the phases
//   Q  fused q|k|v dequant-GEMV of rms(h)                      -> qkv
//   O  o projection of q (+ h)                                 -> h1
//   R  router logits of rms(h1), one gate row per CTA          -> logits
//   D  top-k / softmax / renormalise / unit plan, redundantly in every CTA
//   G  gate|up of the selected experts, SiLU(gate)*up           -> act
//   N  down projection over all units, routing-weighted combine (+ h1) -> h'
//
// Phases hand their outputs to the next phase through small buffers in global
// memory, separated by grid-wide barriers: one red.release per CTA on a counter
// and one acquiring poller per CTA, the fastest all-to-all hand-off measured on
// this part (~1.3 us for 148 CTAs; polling the data words themselves from many
// threads turns the few lines involved into L2 hot spots and is several times
// slower).  Outputs are read back through L2 (ld.global.cg).  Per MoE layer
// there are three barriers (h, logits, act), per clock layer five (+ qkv, h1).
//
// The producer warp walks the same schedule and streams the weight records of the
// CTA's tiles into a shared-memory ring with one bulk copy each: the static
// weights (q|k|v, o, gate rows) are in flight ahead of their phase, the next
// layer's static weights are prefetched into L2 while the router decides, and
// the experts' gate|up and down records are all issued as soon as this CTA has
// built the routing plan.
//
// Numerics follow dq_gemv_kernel (gemv.cu) and route_kernel (moe.cu): offset
// dequantisation ((M + n) in fp16/bf16 straight into mma.sync, fp32 accumulation,
// the exact group correction D - P - z Q applied in fp32 with the group scale),
// logits rounded to the activation dtype, fp32 softmax, ties of the top-k to the
// lower expert id.
#include "gemv_core.cuh"
#include "moe.cuh"
#include "topk.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);

struct StackParams {
  const duplex_stack_layer* layers;
  int n_layers, T, H, E, I, top_k, norm, q_dim, qkv_R, has_attn, moe_residual;
  TileGeom tq, to, tgu, tdn;
  int RbQ, RbO, RbD;
  float rms_eps;
  const void* x_in;
  void* out;
  void* hbuf[2];  // layer input / output h   [T][H] (layer parity)
  void* qkv;      // q|k|v                     [T][qkv_R]
  void* h1;       // h + o(q)                  [T][H]
  float* logits;  // [T][E]
  void* act;      // SiLU(gate)*up            [units][T][I]
  unsigned* barrier;  // grid barrier counter, zeroed before the launch
  int* err;
  int nslots, ups, act_units;
  uint32_t slot_bytes, off_ring, off_x, off_gsum, x_pitch, xd_pitch;
};

// fixed shared-memory map (bytes)
constexpr uint32_t kSFull = 0;        // 16 mbarriers
constexpr uint32_t kSEmpty = 128;     // 16 mbarriers
constexpr uint32_t kSPlan = 256;      // mbarrier: plan of the current layer ready
constexpr uint32_t kSAbort = 272;     // int
constexpr uint32_t kSNUnits = 276;    // int
constexpr uint32_t kSSel = 512;       // [8 tokens][8] ints
constexpr uint32_t kSSelBits = 768;   // [8 tokens][8] words: selected experts
constexpr uint32_t kSUnitE = 1024;    // kMaxUnits ints
constexpr uint32_t kSUnitM = 1280;    // kMaxUnits uints
constexpr uint32_t kSUnitW = 1536;    // kMaxUnits * 8 floats
constexpr uint32_t kSLogit = 3584;    // [8][kMaxExperts] floats
// cross-warp reductions (kCW warps x 2 records x kRedStride floats) and scratch
constexpr int kRedStride = 152;  // swizzled [8 tokens][16 rows] block, see red_at
constexpr uint32_t kSRed = kSLogit + 8 * kMaxExperts * 4;
constexpr uint32_t kSRedBytes = kCW * 2 * kRedStride * 4;
constexpr uint32_t kSFixedEnd = kSRed + kSRedBytes;
constexpr int kSlotsMax = 16;
constexpr int kMaxChunks = 8;  // 8-value chunks of staged rows per consumer thread

// Which wait of this kernel gave up first: err bits from DUPLEX_DEVERR_SITE_SHIFT.
enum : int { kSiteEmpty = 1, kSitePlan = 2, kSiteFull = 3, kSiteGrid = 4, kSiteDrain = 5 };

// Code size matters here: every layer walks all phases, so the per-phase work
// lives in one non-inlined copy each (staging, tile compute, router, plan, the
// barrier, the slow path of the waits) to keep the loop inside the instruction
// cache.
#define DEVN __device__ __noinline__

DEVI void give_up(volatile int* abort, int* err, int site) {
  *abort = 1;
  set_error(err, DUPLEX_DEVERR_TIMEOUT | (site << DUPLEX_DEVERR_SITE_SHIFT));
}

DEVN void wait_phase_slow(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                          int site) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return;
    if (clock64() - t0 > kWaitLimitCycles) {
      give_up(abort, err, site);
      return;
    }
  }
}

// Bounded wait on an mbarrier phase; returns at once when this CTA has given up.
DEVI void wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site) {
  if (*abort || mbar_try_wait(bar, parity)) return;
  wait_phase_slow(bar, parity, abort, err, site);
}

DEVI unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer warps of all CTAs, split into arrival and
// wait so that local work can run in between: the n-th barrier of a launch (n
// from 1) completes when the counter reaches n * gridDim.x.  grid_arrive follows
// a consumer barrier, so the CTA's writes before it are released with the
// arrival (cumulativity), and they are visible to every CTA after grid_wait.
// Bounded: gives up after ~kWaitLimitCycles, or as soon as any CTA has given up.
DEVI void grid_arrive(unsigned* counter) {
  named_bar_sync(1, kConsumers);
  if (threadIdx.x == 0)
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}

DEVN void grid_wait(unsigned* counter, unsigned n, volatile int* abort, int* err) {
  if (threadIdx.x == 0 && !*abort) {
    const unsigned target = n * gridDim.x;
    const long long t0 = clock64();
    int k = 0;
    while ((int)(ld_acquire_gpu(counter) - target) < 0) {
      if ((++k & 63) == 0 && (*reinterpret_cast<volatile int*>(err) & DUPLEX_DEVERR_TIMEOUT)) {
        *abort = 1;
        break;
      }
      if (clock64() - t0 > kWaitLimitCycles) {
        give_up(abort, err, kSiteGrid);
        break;
      }
    }
  }
  named_bar_sync(1, kConsumers);
}

// floor(i / d) for 0 <= i < 2^32 / d, d > 0: one multiply-high with m = fast_div_m(d)
DEVI uint32_t fast_div_m(uint32_t d) { return 0xFFFFFFFFu / d + 1u; }
DEVI uint32_t fast_div(uint32_t i, uint32_t m, uint32_t d) { return d == 1u ? i : __umulhi(i, m); }

// Stage `nrows` rows of K 16-bit values (row r at src + r * row_stride elements,
// read through L2; K % 64 == 0, nrows * K <= 32768) into shared memory in
// fragment order for the offset path (fp16: odd columns / 16), optionally
// RMS-normalised per row (rounded to T) and copied in natural order to
// `plain_out`, and build the correction sums of every `cw` 32-column windows (a
// pair, or a window for group 32): gsum [unit][K / (32 cw)][8 tokens] float2,
// row r = unit * rows_per_unit + token.  `part` is 16 KB of scratch.  Runs on the
// 512 consumer threads; starts and ends with a consumer-wide barrier.
// mode kStageAll does everything; kStageNorm stops after the (normalised)
// natural-order rows are in xsh (and plain_out); kStageFrag takes them from there
// and does the rest (fragment order, correction sums).
enum : int { kStageAll = 0, kStageNorm = 1, kStageFrag = 2 };

template <typename T>
DEVN void stage_rows(const uint8_t* src, int row_stride, int nrows, int K, int rows_per_unit,
                     uint8_t* xsh, uint32_t pitch, bool rms, float eps, uint8_t* plain_out,
                     float2* gsum, int cw, float* part, int mode) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int nq = K >> 3;  // 8-value chunks per row, a multiple of 8
  const int total = nrows * nq;
  const uint32_t mq = fast_div_m((uint32_t)nq), mu = fast_div_m((uint32_t)rows_per_unit);
  // sums of squares: one partial per 32 chunks when rows are whole warps, else
  // per 8 chunks; each row's partials are added in a fixed order (identical run
  // to run)
  const int seg = (nq & 31) == 0 ? 32 : 8;
  named_bar_sync(1, kConsumers);
  // pass 1: fetch into xsh in natural order; sums of squares
  for (int base = 0; mode != kStageFrag && base < total; base += 2 * kConsumers) {
    // both loads of the pair are issued before either is used
    uint4 vv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int idx = base + h * kConsumers + tid;
      vv[h] = make_uint4(0, 0, 0, 0);
      if (idx < total) {
        const int r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq), q = idx - r * nq;
        vv[h] = __ldcg(reinterpret_cast<const uint4*>(src + ((size_t)r * row_stride + q * 8) * 2));
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
    const int idx = base + h * kConsumers + tid;
    const uint4 v = vv[h];
    if (idx < total) {
      const int r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq), q = idx - r * nq;
      *reinterpret_cast<uint4*>(xsh + (uint32_t)r * pitch + (uint32_t)q * 16u) = v;
    }
    if (rms) {
      float a = 0.f;
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) a = fmaf(to_f32<T>(e[k]), to_f32<T>(e[k]), a);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      if (seg == 32) {
        a += __shfl_xor_sync(0xffffffffu, a, 8);
        a += __shfl_xor_sync(0xffffffffu, a, 16);
      }
      if ((lane & (seg - 1)) == 0 && idx < total) part[idx / seg] = a;
    }
    }
  }
  if (mode != kStageFrag) named_bar_sync(1, kConsumers);
  // pass 2: normalise, natural-order copy, fragment order (+ /16), correction sums
  const int cq = 4 * cw;  // chunks per correction unit
  const int Nc = nq / cq;
  for (int base = 0; base < total; base += kConsumers) {
    const int idx = base + tid;
    float se = 0.f, so = 0.f;
    int r = 0, q = 0;
    if (idx < total) {
      r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq);
      q = idx - r * nq;
      uint8_t* cp = xsh + (uint32_t)r * pitch + (uint32_t)q * 16u;
      uint4 o = *reinterpret_cast<const uint4*>(cp);
      if (rms && mode != kStageFrag) {
        const int per = nq / seg;
        const float* pr = part + r * per;
        float a = 0.f;
        for (int c = 0; c < per; ++c) a += pr[c];
        const float sc = 1.0f / sqrtf(a / (float)K + eps);
        T* e = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = from_f32<T>(to_f32<T>(e[k]) * sc);
      }
      if (plain_out && mode != kStageFrag)
        *reinterpret_cast<uint4*>(plain_out + ((size_t)r * K + q * 8) * 2) = o;
      if (mode != kStageNorm) {
        o = to_frag_order(o);
        if (DqOff<T>::kOddDiv16) {
          const __half2 q16 = __float2half2_rn(0.0625f);
          __half2 hy = __hmul2(*reinterpret_cast<__half2*>(&o.y), q16);
          __half2 hw = __hmul2(*reinterpret_cast<__half2*>(&o.w), q16);
          o.y = *reinterpret_cast<uint32_t*>(&hy);
          o.w = *reinterpret_cast<uint32_t*>(&hw);
        }
        // fragment order: e0 = x0, e1 = x4, e2 = x1, e3 = x5, e4 = x2, e5 = x6, e6 = x3, e7 = x7
        const T* e = reinterpret_cast<const T*>(&o);
        se = (to_f32<T>(e[0]) + to_f32<T>(e[1])) + (to_f32<T>(e[4]) + to_f32<T>(e[5]));
        so = (to_f32<T>(e[2]) + to_f32<T>(e[3])) + (to_f32<T>(e[6]) + to_f32<T>(e[7]));
      }
      *reinterpret_cast<uint4*>(cp) = o;
    }
    if (mode == kStageNorm) continue;  // uniform: the same for every thread
    // a correction unit is cq consecutive chunks of one row (aligned lanes)
    se += __shfl_xor_sync(0xffffffffu, se, 1);
    so += __shfl_xor_sync(0xffffffffu, so, 1);
    se += __shfl_xor_sync(0xffffffffu, se, 2);
    so += __shfl_xor_sync(0xffffffffu, so, 2);
    if (cq == 8) {
      se += __shfl_xor_sync(0xffffffffu, se, 4);
      so += __shfl_xor_sync(0xffffffffu, so, 4);
    }
    if (idx < total && (q & (cq - 1)) == 0) {
      const int u = (int)fast_div((uint32_t)r, mu, (uint32_t)rows_per_unit);
      const int n = r - u * rows_per_unit;
      float P, Q;
      if (DqOff<T>::kOddDiv16) {
        P = 1024.f * (se + so);
        Q = fmaf(16.f, so, se);
      } else {
        Q = se + so;
        P = 128.f * Q;
      }
      gsum[((size_t)u * Nc + q / cq) * 8 + n] = make_float2(P, Q);
    }
  }
  named_bar_sync(1, kConsumers);
}

// Cross-warp reduction of one 16-row output tile for NREC records.  Each warp's
// partial (lane (g, t): rows g, g + 8 x tokens 2t, 2t + 1) goes to a swizzled
// [token][row] block, (n, r) at n * 16 + r + (n >> 1) * 8, so that both the
// writes and the readers' column reads are bank-conflict free; only tokens < nT
// are written.  Threads tid < nT * 16 return the sums of row tid & 15, token
// tid >> 4 (record 0 in .x, record 1 in .y).  The caller synchronises before
// `red` is used again.
DEVI int red_at(int n, int r) { return n * 16 + r + (n >> 1) * 8; }
static_assert(7 * 16 + 15 + 3 * 8 < kRedStride, "reduction block");
static_assert(kSRedBytes >= 4 * (kMaxTokens * kMaxExperts + kMaxTokens * kMaxExperts / 4 +
                                   kMaxExperts),
              "scratch users of red: RMS partials, plan keys, candidates, unit_of");

template <int NREC>
DEVI float2 reduce_rows(float* red, const float (&acc)[NREC][4], int nT, int tid, int warp,
                        int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int r = 0; r < NREC; ++r) {
    float* b = red + (warp * NREC + r) * kRedStride;
    if (2 * t < nT) {
      b[red_at(2 * t, g)] = acc[r][0];
      b[red_at(2 * t, g + 8)] = acc[r][2];
    }
    if (2 * t + 1 < nT) {
      b[red_at(2 * t + 1, g)] = acc[r][1];
      b[red_at(2 * t + 1, g + 8)] = acc[r][3];
    }
  }
  named_bar_sync(1, kConsumers);
  float v = 0.f, v2 = 0.f;
  if (tid < nT * 16) {
    const int a = red_at(tid >> 4, tid & 15);
#pragma unroll
    for (int w = 0; w < kCW; ++w) {
      v += red[(w * NREC) * kRedStride + a];
      if (NREC == 2) v2 += red[(w * NREC + 1) * kRedStride + a];
    }
  }
  return make_float2(v, v2);
}

// Accumulators of one lane for up to two records (rows g, g + 8 x tokens 2t, 2t + 1).
struct Acc2 {
  float v[2][4];
};

// One ring stage of NREC records sharing the staged rows: the warp's pair range,
// then the slot is released.  Returns this lane's accumulators.
template <typename T, typename S, int NREC, bool G32>
DEVN Acc2 tile_acc(const uint8_t* st, const TileGeom tg, const uint8_t* xsh, uint32_t pitch,
                   const float2* gsum, int nT, uint64_t* empty_bar) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int np = tg.npairs;
  float acc[NREC][4];
#pragma unroll
  for (int r = 0; r < NREC; ++r) zero4(acc[r]);
  const bool xon = (lane >> 2) < nT;
  if (!G32 && tg.gshift == 1 && np == 2 * kCW)
    pm_fixed<T, S, NREC, 2, 2>(st, tg, warp, lane, xsh, pitch, gsum, xon, acc);
  else if (!G32 && tg.gshift == 1 && np == 4 * kCW)
    pm_fixed<T, S, NREC, 4, 2>(st, tg, warp, lane, xsh, pitch, gsum, xon, acc);
  else
    pm_offset<T, S, NREC, G32>(st, tg, (warp * np) / kCW, ((warp + 1) * np) / kCW, lane, xsh,
                               pitch, gsum, xon, acc);
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);
  Acc2 out;
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int k = 0; k < 4; ++k) out.v[r][k] = r < NREC ? acc[r][k] : 0.f;
  return out;
}

// Deferred cross-warp reduction: the warps' partial sums of up to `rmax` tiles
// wait in `red` ([tile][record][warp][token][row]); one barrier and one pass then
// reduce them all.  Only tokens < nT are kept.
template <int NREC>
DEVI void put_partials(float* red, int jj, const Acc2& a, int nT, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int r = 0; r < NREC; ++r) {
    float* b = red + ((jj * NREC + r) * kCW + warp) * (nT * 16);
    if (2 * t < nT) {
      b[(2 * t) * 16 + g] = a.v[r][0];
      b[(2 * t) * 16 + g + 8] = a.v[r][2];
    }
    if (2 * t + 1 < nT) {
      b[(2 * t + 1) * 16 + g] = a.v[r][1];
      b[(2 * t + 1) * 16 + g + 8] = a.v[r][3];
    }
  }
}

// Sums of output o = jj * nT * 16 + token * 16 + row (records 0 and 1).
template <int NREC>
DEVI float2 sum_partials(const float* red, int o, int nT) {
  const int per = nT * 16;
  const int jj = o / per, rem = o - jj * per;
  float v = 0.f, v2 = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) {
    v += red[((jj * NREC) * kCW + w) * per + rem];
    if (NREC == 2) v2 += red[((jj * NREC + 1) * kCW + w) * per + rem];
  }
  return make_float2(v, v2);
}

// Tiles whose partials fit in `red` at once.
DEVI int defer_tiles(int nrec, int nT) {
  int r = (int)(kSRedBytes / 4) / (nrec * kCW * nT * 16);
  const int by_threads = kConsumers / (nT * 16);
  return r < by_threads ? r : by_threads;
}

// One down-projection stage: `cnt` unit records, each with its own staged rows;
// returns this lane's partial sums (rows g, g + 8 x tokens 2t, 2t + 1).
template <typename T, typename S, bool G32>
DEVN float4 stage_rm(const uint8_t* st, const TileGeom tg, int cnt, const uint8_t* xd,
                     uint32_t xpitch, int nT, const float2* gsum, int ncu, const float* colw,
                     uint64_t* empty_bar) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = cnt * tg.npairs;
  float acc[4];
  zero4(acc);
  const bool xon = (lane >> 2) < nT;
  if (!G32 && tg.gshift == 1 && (tg.npairs & 1) == 0)
    rm_grouped<T, S, 2>(st, tg, cnt, warp, lane, xd, xpitch, nT, gsum, ncu, colw, xon, acc);
  else
    rm_offset<T, S, G32>(st, tg, (warp * items) / kCW, ((warp + 1) * items) / kCW, lane, xd, xpitch,
                         nT, gsum, ncu, colw, xon, acc);
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);
  return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

DEVN float reduce4(float* red, const float4 a, int nT) {
  const int tid = threadIdx.x;
  const float acc[1][4] = {{a.x, a.y, a.z, a.w}};
  return reduce_rows<1>(red, acc, nT, tid, tid >> 5, tid & 31).x;
}

// Router logits of expert e for nT tokens: the gate row (H values, natural order)
// in `wrow`, the normalised tokens in natural order at xrows + n * xpitch.  Thread
// n < nT returns logit n.
template <typename T>
DEVN float router_row(const uint8_t* wrow, const uint8_t* xrows, uint32_t xpitch, int H, int nT,
                      const void* gate_b, int e, float* red, uint64_t* empty_bar) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint4* wr = reinterpret_cast<const uint4*>(wrow);
  const int nq = H >> 3;
  float part[kMaxTokens];
#pragma unroll
  for (int n = 0; n < kMaxTokens; ++n) part[n] = 0.f;
  for (int q = tid; q < nq; q += kConsumers) {
    const uint4 wv = wr[q];
    const T* we = reinterpret_cast<const T*>(&wv);
#pragma unroll
    for (int n = 0; n < kMaxTokens; ++n) {
      if (n < nT) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xrows + (size_t)n * xpitch + (size_t)q * 16);
        const T* xe = reinterpret_cast<const T*>(&xv);
#pragma unroll
        for (int k = 0; k < 8; ++k) part[n] = fmaf(to_f32<T>(we[k]), to_f32<T>(xe[k]), part[n]);
      }
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);
#pragma unroll
  for (int n = 0; n < kMaxTokens; ++n) {
    if (n < nT) {
      float a = part[n];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) red[warp * 8 + n] = a;
    }
  }
  named_bar_sync(1, kConsumers);
  float a = 0.f;
  if (tid < nT) {
#pragma unroll
    for (int w = 0; w < kCW; ++w) a += red[w * 8 + tid];
    if (gate_b) a += to_f32<T>(reinterpret_cast<const T*>(gate_b)[e]);
    a = to_f32<T>(from_f32<T>(a));
  }
  named_bar_sync(1, kConsumers);
  return a;
}

// Router logits with the RMS staging fused in: fetch the nT rows of h (H values,
// through L2), RMS-normalise them in registers (rounded to T), leave them in
// natural order in xsh for the fragment staging that follows, and dot them with
// this CTA's gate row `wrow` (natural order in the ring slot; null when the CTA has
// no router row).  Threads tid < nT return the rounded logit of row tid.  Every
// sum runs in a fixed order.  nT * H <= kMaxChunks * 8 * 512.
template <typename T>
DEVN float router_fused(const uint8_t* src, int H, int nT, bool rms, float eps, uint8_t* xsh,
                        uint32_t pitch, const uint8_t* wrow, const void* gate_b, int e, float* red,
                        uint64_t* empty_bar) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int nq = H >> 3, total = nT * nq;
  const uint32_t mq = fast_div_m((uint32_t)nq);
  const int seg = (nq & 31) == 0 ? 32 : 8;
  const int per = nq / seg;  // segments per row
  float* part = red;         // sums of squares, one per segment
  float* dotp = red + 1024;  // dot products, one per segment
  named_bar_sync(1, kConsumers);
  uint4 v[kMaxChunks];
#pragma unroll
  for (int j = 0; j < kMaxChunks; ++j) {
    const int idx = tid + j * kConsumers;
    v[j] = make_uint4(0, 0, 0, 0);
    if (idx < total) {
      const int r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq), q = idx - r * nq;
      v[j] = __ldcg(reinterpret_cast<const uint4*>(src + ((size_t)r * H + q * 8) * 2));
    }
  }
  if (rms) {
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
      if (j * kConsumers >= total) break;  // uniform
      const int idx = tid + j * kConsumers;
      float a = 0.f;
      const T* x = reinterpret_cast<const T*>(&v[j]);
#pragma unroll
      for (int k = 0; k < 8; ++k) a = fmaf(to_f32<T>(x[k]), to_f32<T>(x[k]), a);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      if (seg == 32) {
        a += __shfl_xor_sync(0xffffffffu, a, 8);
        a += __shfl_xor_sync(0xffffffffu, a, 16);
      }
      if ((lane & (seg - 1)) == 0 && idx < total) part[idx / seg] = a;
    }
    named_bar_sync(1, kConsumers);
  }
#pragma unroll
  for (int j = 0; j < kMaxChunks; ++j) {
    if (j * kConsumers >= total) break;  // uniform
    const int idx = tid + j * kConsumers;
    float d = 0.f;
    if (idx < total) {
      const int r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq), q = idx - r * nq;
      uint4 o = v[j];
      if (rms) {
        float a = 0.f;
        for (int c = 0; c < per; ++c) a += part[r * per + c];
        const float sc = 1.0f / sqrtf(a / (float)H + eps);
        T* x = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = from_f32<T>(to_f32<T>(x[k]) * sc);
      }
      *reinterpret_cast<uint4*>(xsh + (uint32_t)r * pitch + (uint32_t)q * 16u) = o;
      if (wrow) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (size_t)q * 16);
        const T* w = reinterpret_cast<const T*>(&wv);
        const T* x = reinterpret_cast<const T*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) d = fmaf(to_f32<T>(w[k]), to_f32<T>(x[k]), d);
      }
    }
    if (wrow) {
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      if (seg == 32) {
        d += __shfl_xor_sync(0xffffffffu, d, 8);
        d += __shfl_xor_sync(0xffffffffu, d, 16);
      }
      if ((lane & (seg - 1)) == 0 && idx < total) dotp[idx / seg] = d;
    }
  }
  if (wrow) {
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);
  }
  named_bar_sync(1, kConsumers);
  float a = 0.f;
  if (wrow && tid < nT) {
    for (int c = 0; c < per; ++c) a += dotp[tid * per + c];
    if (gate_b) a += to_f32<T>(reinterpret_cast<const T*>(gate_b)[e]);
    a = to_f32<T>(from_f32<T>(a));
  }
  return a;
}

// plan_units for one token: warp 0 alone (lane holds experts lane + 32 i), the same
// keys and max-reductions as the general path, so the same selection; the units are
// the k selected experts in ascending id order (position = number of selected ids
// below).  A function of its own: inside plan_units the general path's code made this
// path ~2.5x slower (3,100 vs 1,250 cycles measured).
template <typename T>
DEVN int plan_one(const float* logits, int E, int top_k, uint8_t* smem, float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* ls = reinterpret_cast<float*>(smem + kSLogit);
  int* sel_s = reinterpret_cast<int*>(smem + kSSel);
  int* unit_e = reinterpret_cast<int*>(smem + kSUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kSUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);
  int* n_units_s = reinterpret_cast<int*>(smem + kSNUnits);
  int* unit_of =  // plan_units's layout of the scratch, read again by plan_weights
      reinterpret_cast<int*>(scratch) + kMaxTokens * kMaxExperts + kMaxTokens * (kMaxExperts / 4);
  (void)tid;
  if (warp == 0) {
    uint32_t key[kMaxExperts / 32];
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      const int e = lane + 32 * i;
      const float v = e < E ? __ldcg(logits + e) : 0.f;
      key[i] = e < E ? order_key<T>(v, e) : 0u;
      if (e < E) ls[e] = v;
    }
    int sel[kMaxTopK];
    int mine = 0;  // lane j's pick
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      sel[j] = 0;
      if (j < top_k) {
        uint32_t lm = 0u;
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i) lm = key[i] > lm ? key[i] : lm;
        const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i)
          if (key[i] == m) key[i] = 0u;
        const int e = key_expert(m);
        sel[j] = (m == 0u || e >= E) ? 0 : e;
        mine = lane == j ? sel[j] : mine;  // taken here: read after the loop, the last pick came out 0
      }
    }
    int rank = 0;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
      if (j < top_k && sel[j] < mine) ++rank;
    if (lane < top_k) {
      sel_s[lane] = mine;
      unit_of[mine] = rank;
      unit_e[rank] = mine;
      unit_m[rank] = 1u;
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) unit_w[rank * kMaxTokens + n] = 0.f;
    }
    if (lane == 0) *n_units_s = top_k;
  }
  named_bar_sync(1, kConsumers);
  return top_k;
}

// Top-k of every token and the unit plan (distinct selected experts in ascending
// id order, their token masks), identical in every CTA.  The routing weights
// follow in plan_weights, off the critical path.  Returns the unit count.
// Top-k by warp max-reductions over the unique keys: per (token, 32-expert block)
// a warp takes the block's top k (k rounds of redux.sync max, the winner's lane
// clears its key), then one warp per token merges the blocks' candidates.
// scratch: keys [T][E] | candidates [T][blocks * top_k] | unit_of [E].
template <typename T>
DEVN int plan_units(const float* logits, int nT, int E, int top_k, uint8_t* smem, float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* ls = reinterpret_cast<float*>(smem + kSLogit);
  int* sel_s = reinterpret_cast<int*>(smem + kSSel);
  int* unit_e = reinterpret_cast<int*>(smem + kSUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kSUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);
  int* n_units_s = reinterpret_cast<int*>(smem + kSNUnits);
  uint32_t* selbits = reinterpret_cast<uint32_t*>(smem + kSSelBits);
  uint32_t* keys = reinterpret_cast<uint32_t*>(scratch);
  const int nblk = (E + 31) >> 5;
  uint32_t* cand = keys + kMaxTokens * kMaxExperts;  // [T][nblk * top_k], every slot written
  int* unit_of = reinterpret_cast<int*>(cand + kMaxTokens * (kMaxExperts / 4));
  const int TE = nT * E;
  for (int idx = tid; idx < TE; idx += kConsumers) {
    const float v = __ldcg(logits + idx);
    const int tk = idx / E;
    ls[idx] = v;
    keys[idx] = order_key<T>(v, idx - tk * E);
  }
  if (tid < kMaxTokens * 8) selbits[tid] = 0u;
  named_bar_sync(1, kConsumers);
  // per (token, block): the block's top k, in descending order
  for (int wu = warp; wu < nT * nblk; wu += kCW) {
    const int tk = wu / nblk, blk = wu - tk * nblk;
    const int e = blk * 32 + lane;
    uint32_t key = e < E ? keys[tk * E + e] : 0u;
    uint32_t* cb = cand + (tk * nblk + blk) * top_k;
    for (int j = 0; j < top_k; ++j) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, key);
      if (key == m && m != 0u) key = 0u;
      if (lane == 0) cb[j] = m;  // 0 once the block has no experts left
    }
  }
  named_bar_sync(1, kConsumers);
  // per token: merge the blocks' candidates (at most 64, two per lane)
  if (warp < nT) {
    const int tk = warp, nc = nblk * top_k;  // <= 64
    uint32_t c0 = lane < nc ? cand[tk * nc + lane] : 0u;
    uint32_t c1 = lane + 32 < nc ? cand[tk * nc + lane + 32] : 0u;
    for (int j = 0; j < top_k; ++j) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, c0 > c1 ? c0 : c1);
      if (m != 0u && c0 == m) c0 = 0u;
      else if (m != 0u && c1 == m) c1 = 0u;
      if (lane == 0) {
        // keys are never 0 and top_k <= E, so m names an expert; clamp regardless
        int e = (int)(0x7FFFu - (m & 0x7FFFu));
        e = (m == 0u || e >= E) ? 0 : e;
        sel_s[tk * 8 + j] = e;
        atomicOr(&selbits[tk * 8 + (e >> 5)], 1u << (e & 31));
      }
    }
  }
  named_bar_sync(1, kConsumers);
  // unit plan: position of a selected expert = selected experts below it
  const int nw = nblk;
  if (warp < nw) {
    const int e = warp * 32 + lane;
    uint32_t mask = 0, below = 0, all = 0;
    for (int w = 0; w < nw; ++w) {
      uint32_t any = 0;
      for (int tk = 0; tk < nT; ++tk) any |= selbits[tk * 8 + w];
      if (w < warp) below += __popc(any);
      all += __popc(any);
      if (w == warp) {
        below += __popc(any & ((1u << lane) - 1u));
        for (int tk = 0; tk < nT; ++tk) mask |= ((selbits[tk * 8 + w] >> lane) & 1u) << tk;
      }
    }
    if (mask) unit_of[e] = below < (uint32_t)kMaxUnits ? (int)below : kMaxUnits;
    if (mask && below < (uint32_t)kMaxUnits) {
      unit_e[below] = e;
      unit_m[below] = mask;
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) unit_w[below * kMaxTokens + n] = 0.f;
    }
    if (tid == 0) *n_units_s = all < (uint32_t)kMaxUnits ? (int)all : kMaxUnits;
  }
  named_bar_sync(1, kConsumers);
  return *n_units_s;
}

// Routing weights of the plan: softmax over all experts, the top-k probabilities
// renormalised (their sum taken in selection order), into unit_w.
DEVN void plan_weights(int nT, int E, int top_k, int norm, uint8_t* smem, const float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* ls = reinterpret_cast<const float*>(smem + kSLogit);
  const int* sel_s = reinterpret_cast<const int*>(smem + kSSel);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);
  const int* unit_of = reinterpret_cast<const int*>(scratch) + kMaxTokens * kMaxExperts +
                       kMaxTokens * (kMaxExperts / 4);
  if (warp < nT) {
    const int tk = warp;
    const float* row = ls + tk * E;
    const float m = row[sel_s[tk * 8]];
    float den = 0.f;
    for (int e = lane; e < E; e += 32) den += expf(row[e] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    const int ej = lane < top_k ? sel_s[tk * 8 + lane] : 0;
    const float pj = lane < top_k ? expf(row[ej] - m) / den : 0.f;
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      const float x = __shfl_sync(0xffffffffu, pj, j);
      if (j < top_k) psum += x;
    }
    if (lane < top_k && ej >= 0 && ej < E) {
      const int u = unit_of[ej];
      if (u >= 0 && u < kMaxUnits) unit_w[u * kMaxTokens + tk] = norm ? pj / psum : pj;
    }
  }
  named_bar_sync(1, kConsumers);
}

DEVI void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

template <typename T, typename S, bool G32>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(const __grid_constant__ StackParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kSEmpty);
  uint64_t* plan_ready = reinterpret_cast<uint64_t*>(smem + kSPlan);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSAbort);
  int* n_units_s = reinterpret_cast<int*>(smem + kSNUnits);
  int* unit_e = reinterpret_cast<int*>(smem + kSUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kSUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nslots;
  const int cta = blockIdx.x, G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], kCW);
    }
    mbar_init(plan_ready, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int perG = p.I >> 4;  // gate|up tiles per unit

  if (warp == kCW) {
    // ================================================================ producer
    const uint64_t pol = policy_evict_first();
    int i = 0;  // stage sequence number
    auto acquire = [&](int j) {
      if (j >= NS)
        wait_phase(&empty[j % NS], (uint32_t)((j / NS) - 1) & 1u, abort_flag, p.err, kSiteEmpty);
    };
    auto slot_ptr = [&](int j) { return smem + p.off_ring + (uint32_t)(j % NS) * p.slot_bytes; };
    // one-copy stage (weights); the second arrival of the full barrier follows at once
    auto issue1 = [&](const uint8_t* src, uint32_t bytes) {
      acquire(i);
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[i % NS], bytes);
        bulk_g2s_stream(slot_ptr(i), src, bytes, &full[i % NS], pol);
        mbar_arrive(&full[i % NS]);
      }
      __syncwarp();
      ++i;
    };

    for (int l = 0; l < p.n_layers; ++l) {
      const duplex_stack_layer L = p.layers[l];
      if (p.has_attn) {
        for (int t = cta; t < p.RbQ; t += G)
          issue1(reinterpret_cast<const uint8_t*>(L.qkv_tiles) + (size_t)t * p.tq.rec_bytes,
                 p.tq.rec_bytes);
        for (int t = cta; t < p.RbO; t += G)
          issue1(reinterpret_cast<const uint8_t*>(L.o_tiles) + (size_t)t * p.to.rec_bytes,
                 p.to.rec_bytes);
      }
      for (int e = cta; e < p.E; e += G)
        issue1(reinterpret_cast<const uint8_t*>(L.gate_w) + (size_t)e * p.H * 2, (uint32_t)p.H * 2u);
      // while the router decides: the next layer's static weights into L2
      if (l + 1 < p.n_layers && lane == 0) {
        const duplex_stack_layer Ln = p.layers[l + 1];
        if (p.has_attn) {
          for (int t = cta; t < p.RbQ; t += G)
            prefetch_l2(reinterpret_cast<const uint8_t*>(Ln.qkv_tiles) + (size_t)t * p.tq.rec_bytes,
                        p.tq.rec_bytes);
          for (int t = cta; t < p.RbO; t += G)
            prefetch_l2(reinterpret_cast<const uint8_t*>(Ln.o_tiles) + (size_t)t * p.to.rec_bytes,
                        p.to.rec_bytes);
        }
        for (int e = cta; e < p.E; e += G)
          prefetch_l2(reinterpret_cast<const uint8_t*>(Ln.gate_w) + (size_t)e * p.H * 2,
                      (uint32_t)p.H * 2u);
      }
      __syncwarp();
      // routing plan of this layer (built by this CTA's consumers)
      wait_phase(plan_ready, (uint32_t)(l & 1), abort_flag, p.err, kSitePlan);
      int nu = *n_units_s;
      nu = nu < 0 ? 0 : (nu > kMaxUnits ? kMaxUnits : nu);
      // never turn an out-of-range id into a copy address
      for (int u = lane; u < nu; u += 32)
        if ((unsigned)unit_e[u] >= (unsigned)p.E) {
          set_error(p.err, DUPLEX_DEVERR_EXPERT);
          unit_e[u] = 0;
        }
      __syncwarp();
      // gate|up: one copy of the (gate, up) record pair per tile
      for (int t = cta; t < nu * perG; t += G) {
        const int u = t / perG, rbi = t - u * perG;
        issue1(reinterpret_cast<const uint8_t*>(L.gu_tiles) +
                   ((size_t)unit_e[u] * (2 * perG) + 2 * rbi) * p.tgu.rec_bytes,
               2u * p.tgu.rec_bytes);
      }
      // down: the records of up to `ups` units per stage, one copy per lane.  Down
      // tiles are dealt from the last CTA backwards, so the CTAs with the fewest
      // gate|up tiles take them first.
      const int nstg = (nu + p.ups - 1) / p.ups;
      for (int t = G - 1 - cta; t < p.RbD; t += G) {
        for (int s = 0; s < nstg; ++s) {
          const int u0 = s * p.ups;
          const int cnt = (nu - u0) < p.ups ? (nu - u0) : p.ups;
          acquire(i);
          if (lane == 0) mbar_arrive_expect_tx(&full[i % NS], (uint32_t)cnt * p.tdn.rec_bytes);
          __syncwarp();
          if (lane < cnt)
            bulk_g2s_stream(slot_ptr(i) + (uint32_t)lane * p.tdn.rec_bytes,
                            reinterpret_cast<const uint8_t*>(L.dn_tiles) +
                                ((size_t)unit_e[u0 + lane] * p.RbD + t) * p.tdn.rec_bytes,
                            p.tdn.rec_bytes, &full[i % NS], pol);
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[i % NS]);
          __syncwarp();
          ++i;
        }
      }
    }
    // drain: never leave the CTA while a bulk copy may still target its smem
    if (lane == 0) {
      const int first = i > NS ? i - NS : 0;
      for (int j = first; j < i; ++j) {
        const long long t0 = clock64();
        bool ok = true;
        while (!mbar_try_wait(&full[j % NS], (uint32_t)(j / NS) & 1u))
          if (clock64() - t0 > 200000000LL) {
            ok = false;
            break;
          }
        if (!ok) {
          give_up(abort_flag, p.err, kSiteDrain);
          break;
        }
      }
    }
    return;
  }

  // ================================================================== consumers
  float* red = reinterpret_cast<float*>(smem + kSRed);
  uint8_t* xsh = smem + p.off_x;
  float2* gsum = reinterpret_cast<float2*>(smem + p.off_gsum);
  const int nT = p.T;
  const int cw = G32 ? 1 : 2;
  int* err = p.err;
  int i = 0;       // stage sequence number
  unsigned nb = 0;  // grid barriers passed

  auto wait_full = [&](int j) {
    wait_phase(&full[j % NS], (uint32_t)(j / NS) & 1u, abort_flag, err, kSiteFull);
  };
  auto slot_ptr = [&](int j) { return smem + p.off_ring + (uint32_t)(j % NS) * p.slot_bytes; };
  auto sync_grid = [&]() {
    grid_arrive(p.barrier);
    grid_wait(p.barrier, ++nb, abort_flag, err);
  };

  for (int l = 0; l < p.n_layers; ++l) {
    const duplex_stack_layer L = p.layers[l];
    const bool last = l == p.n_layers - 1;
    const T* hin = reinterpret_cast<const T*>(l == 0 ? p.x_in : p.hbuf[l & 1]);
    T* hout = reinterpret_cast<T*>(last ? p.out : p.hbuf[(l + 1) & 1]);
    const T* hm = hin;  // MoE input
    if (p.has_attn) {
      // ---------------------------------------------------------------- Q
      stage_rows<T>(reinterpret_cast<const uint8_t*>(hin), p.H, nT, p.H, nT, xsh, p.x_pitch,
                    p.rms_eps > 0.f, p.rms_eps, nullptr, gsum, cw, red, kStageAll);
      {
        const int rmax = defer_tiles(1, nT);
        int j = 0, t0 = cta;
        for (int tile = cta; tile < p.RbQ; tile += G, ++i) {
          wait_full(i);
          const Acc2 a = tile_acc<T, S, 1, G32>(slot_ptr(i), p.tq, xsh, p.x_pitch, gsum, nT,
                                                &empty[i % NS]);
          put_partials<1>(red, j++, a, nT, warp, lane);
          if (j == rmax || tile + G >= p.RbQ) {
            named_bar_sync(1, kConsumers);
            if (tid < j * nT * 16) {
              const float v = sum_partials<1>(red, tid, nT).x;
              const int jj = tid / (nT * 16), n = (tid >> 4) - jj * nT;
              const int row = (t0 + jj * G) * 16 + (tid & 15);
              reinterpret_cast<T*>(p.qkv)[(size_t)n * p.qkv_R + row] = from_f32<T>(v);
            }
            named_bar_sync(1, kConsumers);
            j = 0;
            t0 = tile + G;
          }
        }
      }
      sync_grid();
      // ---------------------------------------------------------------- O
      if (cta < p.RbO)
        stage_rows<T>(reinterpret_cast<const uint8_t*>(p.qkv), p.qkv_R, nT, p.q_dim, nT, xsh,
                      p.x_pitch, false, 0.f, nullptr, gsum, cw, red, kStageAll);
      {
        const int rmax = defer_tiles(1, nT);
        int j = 0, t0 = cta;
        for (int tile = cta; tile < p.RbO; tile += G, ++i) {
          wait_full(i);
          const Acc2 a = tile_acc<T, S, 1, G32>(slot_ptr(i), p.to, xsh, p.x_pitch, gsum, nT,
                                                &empty[i % NS]);
          put_partials<1>(red, j++, a, nT, warp, lane);
          if (j == rmax || tile + G >= p.RbO) {
            named_bar_sync(1, kConsumers);
            if (tid < j * nT * 16) {
              const float v = sum_partials<1>(red, tid, nT).x;
              const int jj = tid / (nT * 16), n = (tid >> 4) - jj * nT;
              const int row = (t0 + jj * G) * 16 + (tid & 15);
              const float res = to_f32<T>(__ldcg(hin + (size_t)n * p.H + row));
              reinterpret_cast<T*>(p.h1)[(size_t)n * p.H + row] =
                  from_f32<T>(to_f32<T>(from_f32<T>(v)) + res);
            }
            named_bar_sync(1, kConsumers);
            j = 0;
            t0 = tile + G;
          }
        }
      }
      sync_grid();
      hm = reinterpret_cast<const T*>(p.h1);
    }
    // ------------------------------------------------------------------ R
    // normalised rows and this CTA's logit first; their fragment-order staging for
    // the gate|up tiles runs while the logits barrier is in flight
    {
      const bool row = cta < p.E;
      if (row) wait_full(i);
      const float a = router_fused<T>(reinterpret_cast<const uint8_t*>(hm), p.H, nT, p.rms_eps > 0.f,
                                      p.rms_eps, xsh, p.x_pitch, row ? slot_ptr(i) : nullptr,
                                      L.gate_b, cta, red, &empty[i % NS]);
      if (row) {
        if (tid < nT) p.logits[(size_t)tid * p.E + cta] = a;
        ++i;
      }
      for (int e = cta + G; e < p.E; e += G, ++i) {  // more experts than CTAs
        wait_full(i);
        const float a2 = router_row<T>(slot_ptr(i), xsh, p.x_pitch, p.H, nT, L.gate_b, e, red,
                                       &empty[i % NS]);
        if (tid < nT) p.logits[(size_t)tid * p.E + e] = a2;
      }
    }
    grid_arrive(p.barrier);
    stage_rows<T>(nullptr, 0, nT, p.H, nT, xsh, p.x_pitch, false, 0.f, nullptr, gsum, cw, red,
                  kStageFrag);
    grid_wait(p.barrier, ++nb, abort_flag, err);
    // ------------------------------------------------------------------ D
    const int nu = nT == 1 ? plan_one<T>(p.logits, p.E, p.top_k, smem, red)
                           : plan_units<T>(p.logits, nT, p.E, p.top_k, smem, red);
    if (tid == 0) mbar_arrive(plan_ready);
    plan_weights(nT, p.E, p.top_k, p.norm, smem, red);
    // ------------------------------------------------------------------ G
    {
      const int rmax = defer_tiles(2, nT);
      int j = 0, t0 = cta;
      for (int tile = cta; tile < nu * perG; tile += G, ++i) {
        wait_full(i);
        const Acc2 a = tile_acc<T, S, 2, G32>(slot_ptr(i), p.tgu, xsh, p.x_pitch, gsum, nT,
                                              &empty[i % NS]);
        put_partials<2>(red, j++, a, nT, warp, lane);
        if (j == rmax || tile + G >= nu * perG) {
          named_bar_sync(1, kConsumers);
          if (tid < j * nT * 16) {
            const float2 v = sum_partials<2>(red, tid, nT);
            const int jj = tid / (nT * 16), n = (tid >> 4) - jj * nT;
            const int tl = t0 + jj * G;
            const int u = tl / perG, row = (tl - u * perG) * 16 + (tid & 15);
            const float a = ((unit_m[u] >> n) & 1u) ? silu_f32(v.x) * v.y : 0.f;
            reinterpret_cast<T*>(p.act)[((size_t)u * nT + n) * p.I + row] = from_f32<T>(a);
          }
          named_bar_sync(1, kConsumers);
          j = 0;
          t0 = tile + G;
        }
      }
    }
    sync_grid();
    // ------------------------------------------------------------------ N
    const int nstg = (nu + p.ups - 1) / p.ups;
    const int ncu = p.tdn.npairs * (G32 ? 2 : 1);  // correction units per record
    int a0 = -1, acnt = 0;                         // staged activation units [a0, a0 + acnt)
    for (int tile = G - 1 - cta; tile < p.RbD; tile += G) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < nstg; ++s, ++i) {
        const int u0 = s * p.ups;
        const int cnt = (nu - u0) < p.ups ? (nu - u0) : p.ups;
        if (a0 < 0 || u0 < a0 || u0 + cnt > a0 + acnt) {
          a0 = u0;
          acnt = (nu - u0) < p.act_units ? (nu - u0) : p.act_units;
          stage_rows<T>(reinterpret_cast<const uint8_t*>(p.act) + (size_t)a0 * nT * p.I * 2, p.I,
                        acnt * nT, p.I, nT, xsh, p.xd_pitch, false, 0.f, nullptr, gsum, cw, red,
                        kStageAll);
        }
        wait_full(i);
        const float4 d = stage_rm<T, S, G32>(slot_ptr(i), p.tdn, cnt,
                                             xsh + (uint32_t)((u0 - a0) * nT) * p.xd_pitch,
                                             p.xd_pitch, nT, gsum + (size_t)(u0 - a0) * ncu * 8, ncu,
                                             unit_w + u0 * kMaxTokens, &empty[i % NS]);
        acc.x += d.x;
        acc.y += d.y;
        acc.z += d.z;
        acc.w += d.w;
      }
      const float v = reduce4(red, acc, nT);
      if (tid < nT * 16) {
        const int n = tid >> 4, row = tile * 16 + (tid & 15);
        float y = v;
        if (p.moe_residual) y += to_f32<T>(__ldcg(hm + (size_t)n * p.H + row));
        hout[(size_t)n * p.H + row] = from_f32<T>(y);
      }
      named_bar_sync(1, kConsumers);
    }
    if (!last) sync_grid();
  }
}

// ====================================================================== host side
static inline uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct StackScratch {
  size_t barrier, hbuf[2], qkv, h1, logits, act, total;
};

static int units_cap(int T, int E, int top_k) {
  int units = T * top_k < E ? T * top_k : E;
  return units > kMaxUnits ? kMaxUnits : units;
}

static StackScratch stack_scratch(int T, int H, int E, int I, int top_k, int qkv_R) {
  StackScratch s;
  size_t off = 0;
  s.barrier = off;
  off += 256;
  for (int k = 0; k < 2; ++k) {
    s.hbuf[k] = off;
    off += align_up((size_t)T * H * 2, 256);
  }
  s.qkv = off;
  off += align_up((size_t)T * (qkv_R > 0 ? qkv_R : 1) * 2, 256);
  s.h1 = off;
  off += align_up((size_t)T * H * 2, 256);
  s.logits = off;
  off += align_up((size_t)T * E * 4, 256);
  s.act = off;
  off += align_up((size_t)units_cap(T, E, top_k) * T * I * 2, 256);
  s.total = off;
  return s;
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_stack_workspace_bytes(int32_t T, int32_t H, int32_t E, int32_t I,
                                            int32_t top_k, int32_t qkv_R, size_t* bytes) {
  if (!bytes || T < 1 || H < 1 || E < 1 || I < 1 || top_k < 1) return DUPLEX_ERR_ARG;
  *bytes = stack_scratch(T, H, E, I, top_k, qkv_R).total;
  return DUPLEX_OK;
}

extern "C" int duplex_stack_forward(const duplex_stack_layer* layers, int32_t n_layers,
                                    int32_t has_attn, int32_t moe_residual, const void* x_in,
                                    void* out, int act_dtype, int scale_dtype, int has_zeros,
                                    int32_t T, int32_t H, int32_t E, int32_t I, int32_t top_k,
                                    int32_t norm_topk, int32_t qkv_R, int32_t q_dim,
                                    int32_t group, float rms_eps, void* workspace,
                                    size_t workspace_bytes, int32_t* err, void* stream) {
  if (!layers || n_layers < 1 || n_layers > 255 || !x_in || !out || !workspace || !err)
    return DUPLEX_ERR_ARG;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  if ((H & 63) || (I & 63) || group < 32 || (group & (group - 1))) return DUPLEX_ERR_UNSUPPORTED;
  StackParams p = {};
  if (tile_geom(H, group, has_zeros, &p.tgu) || tile_geom(I, group, has_zeros, &p.tdn))
    return DUPLEX_ERR_UNSUPPORTED;
  p.has_attn = has_attn ? 1 : 0;
  if (p.has_attn) {
    if (qkv_R < 16 || (qkv_R & 15) || q_dim < 64 || (q_dim & 63) || q_dim > qkv_R)
      return DUPLEX_ERR_UNSUPPORTED;
    if (tile_geom(H, group, has_zeros, &p.tq) || tile_geom(q_dim, group, has_zeros, &p.to))
      return DUPLEX_ERR_UNSUPPORTED;
  }
  const int G = num_sms();
  const StackScratch L = stack_scratch(T, H, E, I, top_k, p.has_attn ? qkv_R : 0);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(x_in) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return DUPLEX_ERR_ALIGN;
  // staged rows must fit the per-thread chunk registers
  const int maxK = p.has_attn && q_dim > H ? q_dim : H;
  if (T * maxK > kMaxChunks * 8 * kConsumers) return DUPLEX_ERR_UNSUPPORTED;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  p.layers = layers;
  p.n_layers = n_layers;
  p.T = T; p.H = H; p.E = E; p.I = I; p.top_k = top_k; p.norm = norm_topk;
  p.q_dim = q_dim; p.qkv_R = qkv_R; p.moe_residual = moe_residual ? 1 : 0;
  p.RbQ = (qkv_R + 15) / 16; p.RbO = (H + 15) / 16; p.RbD = (H + 15) / 16;
  p.rms_eps = rms_eps;
  p.x_in = x_in; p.out = out;
  for (int k = 0; k < 2; ++k) p.hbuf[k] = ws + L.hbuf[k];
  p.qkv = ws + L.qkv;
  p.h1 = ws + L.h1;
  p.logits = reinterpret_cast<float*>(ws + L.logits);
  p.act = ws + L.act;
  p.barrier = reinterpret_cast<unsigned*>(ws + L.barrier);
  p.err = err;
  // ring slot: the largest stage -- a q|k|v record, an o record, a gate row, or a
  // gate|up record pair; down stages take as many unit records as fit
  uint32_t slot = 2u * p.tgu.rec_bytes;
  if (p.has_attn) {
    slot = slot > p.tq.rec_bytes ? slot : p.tq.rec_bytes;
    slot = slot > p.to.rec_bytes ? slot : p.to.rec_bytes;
  }
  slot = slot > (uint32_t)H * 2u ? slot : (uint32_t)H * 2u;
  if (slot < p.tdn.rec_bytes) slot = p.tdn.rec_bytes;
  slot = up(slot, 128);
  int ups = (int)(slot / p.tdn.rec_bytes);
  if (ups > 32) ups = 32;
  // activation units staged at once for the down projection (at least one stage)
  const int by_regs = (kMaxChunks * 8 * kConsumers) / (T * I);
  if (by_regs < 1) return DUPLEX_ERR_UNSUPPORTED;
  if (ups > by_regs) ups = by_regs;
  const int ucap = units_cap(T, E, top_k);
  int act_units = ucap < by_regs ? ucap : by_regs;
  if (act_units < ups) act_units = ups;
  p.ups = ups;
  p.act_units = act_units;
  p.slot_bytes = slot;
  p.x_pitch = up((uint32_t)((maxK + 63) / 64 * 64) * 2u, 128) + 64u;
  p.xd_pitch = up((uint32_t)I * 2u, 128) + 64u;
  const uint32_t x_bytes_q = (uint32_t)T * p.x_pitch;
  const uint32_t x_bytes_d = (uint32_t)(act_units * T) * p.xd_pitch;
  const uint32_t x_bytes = x_bytes_q > x_bytes_d ? x_bytes_q : x_bytes_d;
  const int gs_q = (maxK / 32) * 8, gs_d = act_units * (I / 32) * 8;
  const uint32_t gsum_bytes = (uint32_t)((gs_q > gs_d ? gs_q : gs_d) * 8);
  p.off_gsum = up(kSFixedEnd, 128);
  p.off_x = up(p.off_gsum + gsum_bytes, 128);
  p.off_ring = up(p.off_x + x_bytes, 128);
  const size_t kMax = 227 * 1024;
  int ns = p.off_ring < kMax ? (int)((kMax - p.off_ring) / slot) : 0;
  if (ns > kSlotsMax) ns = kSlotsMax;
  if (ns < 2) return DUPLEX_ERR_UNSUPPORTED;
  p.nslots = ns;
  const size_t smem = p.off_ring + (size_t)ns * slot;

  cudaStream_t st = (cudaStream_t)stream;
  const bool g32 = group == 32;
  void (*kern)(StackParams);
  if (act_dtype == DUPLEX_DTYPE_F16)
    kern = g32 ? stack_kernel<__half, __half, true> : stack_kernel<__half, __half, false>;
  else
    kern = g32 ? stack_kernel<__nv_bfloat16, __nv_bfloat16, true>
               : stack_kernel<__nv_bfloat16, __nv_bfloat16, false>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kMax);
  if (rc) return rc;
  int occ = 0;
  rc = record_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));
  if (rc) return rc;
  if (occ < 1) return DUPLEX_ERR_UNSUPPORTED;
  rc = record_cuda(cudaMemsetAsync(ws + L.barrier, 0, 256, st));
  if (rc) return rc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, p));
}
