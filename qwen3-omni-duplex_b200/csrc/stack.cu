// Persistent clock-path kernel on thread-block clusters: every int4 linear of L
// Thinker layers for T <= 8 decode tokens in ONE launch.
//
// The grid is C clusters of kCS = 8 CTAs (one CTA per SM, 16 consumer warps + one
// producer warp).  A decode MoE layer runs
//
//   input    the layer input h = the previous layer's output, which every CTA added
//            into a fixed-point accumulator (+ residual), read by every CTA after the
//            grid barrier, with its RMS scale
//   router   each CTA of a cluster computes E / 8 logits from gate rows that were
//            streamed into its shared memory during the previous layer, and sends
//            them to the cluster (DSMEM)
//   plan     top-k / softmax / renormalise / unit plan, identical in every CTA
//   items    the cluster's share of the (selected expert, 128-column slice of the
//            intermediate) items: CTA r computes gate|up rows [16 r, 16 r + 16) of
//            the slice, SiLU(gate) * up, and sends them to the cluster (DSMEM); then
//            every CTA multiplies the slice's 128 intermediate values by the matching
//            128 columns of the expert's down weights for its H / 8 output rows,
//            weighted by the routing weight, accumulating in registers
//   end      each CTA adds its rows of the cluster's partial output into the layer's
//            fixed-point accumulator (red.global.add of int64: order-independent, so
//            bit-identical) and arrives on the grid barrier
//
// so a MoE layer has ONE grid-wide barrier; every other hand-off stays inside a
// cluster (mbarriers with cluster-scope release / acquire).  A clock layer adds the
// fused q|k|v and the o projection, each followed by a grid barrier (their outputs
// are needed by every CTA).
//
// The producer warp streams each stage (one bulk copy into a shared-memory ring):
// the static weights of a layer (q|k|v and o tiles, this CTA's gate rows) as soon
// as ring slots free up -- i.e. while the previous layer's experts are consumed --
// and the experts' gate|up tile pairs and down K-slice records as soon as this CTA
// has built the routing plan.
//
// Numerics follow dq_gemv_kernel (gemv.cu) and route_kernel (moe.cu): offset
// dequantisation ((M + n) in fp16/bf16 straight into mma.sync, fp32 accumulation,
// the exact group correction D - P - z Q applied in fp32 with the group scale),
// logits rounded to the activation dtype, fp32 softmax, ties of the top-k to the
// lower expert id.  Every sum runs in a fixed order, so launches are bit-identical.
#include "gemv_core.cuh"
#include "moe.cuh"
#include "topk.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);

constexpr int kCS = 8;            // CTAs per cluster
constexpr int kMaxClusters = 32;  // partial-sum slots in the workspace
constexpr int kSliceK = 128;      // intermediate columns per item (kCS gate|up tiles of 16 rows)
static_assert(kSliceK == 16 * kCS, "one gate|up tile per CTA of a cluster per item");
constexpr int kMaxRecPerWarp = 2; // down records (16 output rows) per warp: H <= 4096
constexpr uint32_t kXdPitch = 320;  // bytes per token row of a staged slice (conflict-free)

struct StackParams {
  const duplex_stack_layer* layers;
  int n_layers, T, H, E, I, top_k, norm, q_dim, qkv_R, has_attn, moe_residual;
  TileGeom tq, to, tgu, tks;  // q|k|v, o, gate|up tiles; down K-slice records
  int RbQ, RbO;
  int S;      // down K-slices per expert (I / kSliceK)
  int rrows;  // output rows of the down projection per CTA (H / kCS)
  int nblk;   // 16-expert blocks of the gate records
  int KS;     // 16-column k-steps of a gate block (H / 16)
  int kps;    // k-steps per gate ring stage
  float rms_eps;
  const void* x_in;
  void* out;
  unsigned long long* acc;  // [3][T][H] fixed-point layer outputs (see add_partials)
  void* qkv;    // q|k|v [T][qkv_R]
  void* h1;     // h + o(q) [T][H]
  unsigned* barrier;  // grid barrier counter, zeroed before the launch
  int* err;
  long long wait_limit;
  int test_flags;
  int nslots;
  int ib;             // items per batch
  uint32_t dn_bytes;  // a CTA's down records of one item
  uint32_t slot_bytes, off_ring, off_x, off_gsum, off_h, off_xd, off_av, off_dg, x_pitch;
};

// fixed shared-memory map (bytes)
constexpr uint32_t kSFull = 0;        // 16 mbarriers
constexpr uint32_t kSEmpty = 128;     // 16 mbarriers
constexpr uint32_t kSPlan = 256;      // mbarrier: plan of the current layer ready (producer)
constexpr uint32_t kSHx = 264;        // (free)
constexpr uint32_t kSLg = 272;        // mbarrier: logits of the cluster arrived
constexpr uint32_t kSAct = 280;       // 2 mbarriers: intermediate slices arrived
constexpr uint32_t kSAbort = 296;     // int
constexpr uint32_t kSNUnits = 300;    // int
constexpr uint32_t kSSsq = 320;       // (free)
constexpr uint32_t kSSel = 576;       // [8 tokens][8] ints
constexpr uint32_t kSSelBits = 832;   // [8 tokens][8] words: selected experts
constexpr uint32_t kSUnitE = 1088;    // kMaxUnits ints
constexpr uint32_t kSUnitM = 1344;    // kMaxUnits uints
constexpr uint32_t kSUnitW = 1600;    // kMaxUnits * 8 floats
constexpr uint32_t kSLogit = 3648;    // [8 tokens][kMaxExperts] floats
constexpr uint32_t kSInv = 11840;     // [8] floats: RMS scale per token
// cross-warp reductions (kCW warps x 2 records x kRedStride floats) and scratch
constexpr int kRedStride = 152;  // swizzled [8 tokens][16 rows] block, see red_at
constexpr uint32_t kSRed = 11904;
constexpr uint32_t kSRedBytes = kCW * 2 * kRedStride * 4;
constexpr uint32_t kSFixedEnd = kSRed + kSRedBytes;
static_assert(kSSel >= kSSsq + kCS * 8 * 4, "smem map");
static_assert(kSInv >= kSLogit + 8 * kMaxExperts * 4, "smem map");
static_assert(kSRed % 128 == 0 && kSRed >= kSInv + 32, "smem map");
constexpr int kMaxBatch = 4;      // items of a CTA processed together (one exchange)
constexpr int kMaxBatchRows = 32; // batch items x tokens: staged intermediate rows per buffer
constexpr int kSlotsMax = 16;
constexpr int kMaxChunks = 8;  // 8-value chunks of staged rows per consumer thread

// Which wait of this kernel gave up first: err bits from DUPLEX_DEVERR_SITE_SHIFT.
enum : int {
  kSiteEmpty = 1, kSitePlan = 2, kSiteFull = 3, kSiteGrid = 4, kSiteDrain = 5, kSiteCluster = 6
};

// Code size and calls both cost here.  The phases on the per-item path (the tile
// loops, the exchanges, the router) are inlined: a call saves live registers to
// the stack, and with ~227 KB of shared memory the L1 left for that local memory is
// small (measured: 21.7 -> 18.6 us per MoE layer).  The once-per-layer phases stay
// in one non-inlined copy each, to keep the layer loop inside the instruction cache.
#define DEVN __device__ __noinline__

// Position in the ring of stage buffers: slot and the parity of its use, advanced
// stage by stage (no division per stage).
struct RingPos {
  int slot;
  uint32_t phase;
  DEVI void next(int ns) {
    if (++slot == ns) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// ------------------------------------------------------------------ cluster PTX
DEVI uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
DEVI uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
DEVI uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// address of the same shared-memory location in CTA `rank` of this cluster
DEVI uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
DEVI void st_peer_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
DEVI void st_peer_v2(uint32_t addr, uint2 v) {
  asm volatile("st.shared::cluster.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(v.x), "r"(v.y)
               : "memory");
}
DEVI void st_peer_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
DEVI void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
// one arrival on the mbarrier at cluster shared address `addr`, releasing this
// thread's (and, through the preceding CTA barrier, its CTA's) earlier writes
DEVI void mbar_arrive_peer(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr)
               : "memory");
}
DEVI bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// all threads of all CTAs of the cluster (every thread of the CTA executes it)
DEVI void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ------------------------------------------------------------------ bounded waits
// Give up: stop this CTA's waits and record DUPLEX_DEVERR_TIMEOUT; the first wait
// of the launch that gives up also records its site.
DEVI void give_up(volatile int* abort, int* err, int site) {
  *abort = 1;
  const int old = atomicOr(err, DUPLEX_DEVERR_TIMEOUT);
  if (((old >> DUPLEX_DEVERR_SITE_SHIFT) & 0xFF) == 0)
    atomicCAS(err, old | DUPLEX_DEVERR_TIMEOUT,
              old | DUPLEX_DEVERR_TIMEOUT | (site << DUPLEX_DEVERR_SITE_SHIFT));
}

DEVN void wait_phase_slow(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site,
                          long long limit, bool cluster) {
  const long long t0 = clock64();
  while (!(cluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity))) {
    if (*abort) return;
    if (clock64() - t0 > limit) {
      give_up(abort, err, site);
      return;
    }
  }
}

// Bounded wait on an mbarrier phase; returns at once when this CTA has given up.
DEVI void wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site,
                     long long limit) {
  if (*abort || mbar_try_wait(bar, parity)) return;
  wait_phase_slow(bar, parity, abort, err, site, limit, false);
}

// Bounded wait of the consumers on a cluster exchange: thread 0 waits (acquire at
// cluster scope), then the consumer barrier publishes the data to the CTA.
DEVI void wait_cluster_xchg(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                            long long limit) {
  if (threadIdx.x == 0 && !*abort && !mbar_try_wait_cluster(bar, parity))
    wait_phase_slow(bar, parity, abort, err, kSiteCluster, limit, true);
  named_bar_sync(1, kConsumers);
}

// After this CTA's consumers wrote their part of an exchange into every CTA of the
// cluster: one arrival on `bar` of each CTA (the consumer barrier orders the writes
// of all threads before the arriving threads' releases).
DEVI void signal_cluster_xchg(uint64_t* bar) {
  named_bar_sync(1, kConsumers);
  // thread q arrives on CTA q's barrier: each release is a fence of its own, so the
  // eight run in parallel rather than one after another
  if (threadIdx.x < kCS) mbar_arrive_peer(peer_addr(bar, threadIdx.x));
}

DEVI unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer warps of all CTAs, split into arrival and
// wait: the n-th barrier of a launch (n from 1) completes when the counter reaches
// n * gridDim.x (+ 1 with `unreachable`, which only the timeout test asks for).
// grid_arrive follows a consumer barrier, so the CTA's writes before it are
// released with the arrival.  Bounded: gives up after `limit` cycles, or as soon
// as any CTA has given up.
DEVI void grid_arrive(unsigned* counter) {
  named_bar_sync(1, kConsumers);
  if (threadIdx.x == 0)
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}

DEVN void grid_wait(unsigned* counter, unsigned n, bool unreachable, volatile int* abort, int* err,
                    long long limit) {
  if (threadIdx.x == 0 && !*abort) {
    const unsigned target = n * gridDim.x + (unreachable ? 1u : 0u);
    const long long t0 = clock64();
    int k = 0;
    while ((int)(ld_acquire_gpu(counter) - target) < 0) {
      if ((++k & 63) == 0 && (*reinterpret_cast<volatile int*>(err) & DUPLEX_DEVERR_TIMEOUT)) {
        *abort = 1;
        break;
      }
      if (clock64() - t0 > limit) {
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
// read through L2; K % 64 == 0) into shared memory in fragment order for the
// offset path (fp16: odd columns / 16) and build the correction sums of every `cw`
// 32-column windows: gsum [K / (32 cw)][8 tokens] float2.  `part` is scratch.  Runs
// on the 512 consumer threads; starts and ends with a consumer-wide barrier.
// mode kStageAll fetches from src; kStageFrag takes natural-order rows already in
// xsh and converts them in place.
enum : int { kStageAll = 0, kStageFrag = 2 };

template <typename T>
DEVN void stage_rows(const uint8_t* src, int row_stride, int nrows, int K, uint8_t* xsh,
                     uint32_t pitch, float2* gsum, int cw, int mode) {
  const int tid = threadIdx.x;
  const int nq = K >> 3;  // 8-value chunks per row, a multiple of 8
  const int total = nrows * nq;
  const uint32_t mq = fast_div_m((uint32_t)nq);
  named_bar_sync(1, kConsumers);
  for (int base = 0; mode != kStageFrag && base < total; base += 2 * kConsumers) {
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
      if (idx < total) {
        const int r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq), q = idx - r * nq;
        *reinterpret_cast<uint4*>(xsh + (uint32_t)r * pitch + (uint32_t)q * 16u) = vv[h];
      }
    }
  }
  if (mode != kStageFrag) named_bar_sync(1, kConsumers);
  const int cq = 4 * cw;  // chunks per correction unit
  for (int base = 0; base < total; base += kConsumers) {
    const int idx = base + tid;
    float se = 0.f, so = 0.f;
    int r = 0, q = 0;
    if (idx < total) {
      r = (int)fast_div((uint32_t)idx, mq, (uint32_t)nq);
      q = idx - r * nq;
      uint8_t* cp = xsh + (uint32_t)r * pitch + (uint32_t)q * 16u;
      uint4 o = to_frag_order(*reinterpret_cast<const uint4*>(cp));
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
      *reinterpret_cast<uint4*>(cp) = o;
    }
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
      float P, Q;
      if (DqOff<T>::kOddDiv16) {
        P = 1024.f * (se + so);
        Q = fmaf(16.f, so, se);
      } else {
        Q = se + so;
        P = 128.f * Q;
      }
      gsum[(size_t)(q / cq) * 8 + r] = make_float2(P, Q);
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
              "scratch users of red: plan keys, candidates, unit_of");

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

// One ring stage of NREC records sharing the staged rows: the warp's pair range,
// then the slot is released and the warp's partial sums go to `red` as deferred
// tile jj ([jj][record][warp][token][row], tokens < nT only).
template <typename T, typename S, int NREC, bool G32>
DEVI void tile_acc(const uint8_t* st, const TileGeom tg, const uint8_t* xsh, uint32_t pitch,
                   const float2* gsum, int nT, uint64_t* empty_bar, float* red, int jj) {
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
  // the warp's partial sums, deferred: red [jj][record][warp][token][row]
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int r = 0; r < NREC; ++r) {
    float* b = red + ((jj * NREC + r) * kCW + warp) * (nT * 16);
    if (2 * t < nT) {
      b[(2 * t) * 16 + g] = acc[r][0];
      b[(2 * t) * 16 + g + 8] = acc[r][2];
    }
    if (2 * t + 1 < nT) {
      b[(2 * t + 1) * 16 + g] = acc[r][1];
      b[(2 * t + 1) * 16 + g + 8] = acc[r][3];
    }
  }
}


// Sum of output o = jj * nT * 16 + token * 16 + row.
DEVI float sum_partials(const float* red, int o, int nT) {
  const int per = nT * 16;
  const int jj = o / per, rem = o - jj * per;
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) v += red[(jj * kCW + w) * per + rem];
  return v;
}

// Tiles whose partials fit in `red` at once.
DEVI int defer_tiles(int nT) {
  int r = (int)(kSRedBytes / 4) / (kCW * nT * 16);
  const int by_threads = kConsumers / (nT * 16);
  return r < by_threads ? r : by_threads;
}

// ------------------------------------------------------------------ h exchange
// The clusters' partial layer outputs meet in a fixed-point accumulator: every CTA adds
// its rows' partial sums, scaled by 2^32 and rounded to int64, with red.global.add
// (add_partials).  Integer addition is associative, so the sum is the same bits
// whatever order the 15 clusters' adds land in: no partial buffers, no cross-cluster
// reduction pass, and bit-identical launches.  Partials are clamped to +-2^26 (beyond
// the fp16 range; a clamped or NaN partial sets DUPLEX_DEVERR_NONFINITE), so the sum of
// up to 32 clusters stays inside int64; below 2^-9 a partial keeps 2^-33 absolute
// resolution, finer than any fp16 / bf16 output needs.
constexpr float kFixScale = 4294967296.0f;           // 2^32
constexpr float kFixInv = 2.3283064365386963e-10f;   // 2^-32
constexpr float kFixClamp = 67108864.0f;             // 2^26
static_assert(kMaxClusters * kCS <= 256, "fixed-point sum of every CTA's partial fits int64");

DEVI unsigned long long to_fix(float v, int* err) {
  if (!(fabsf(v) <= kFixClamp)) {
    set_error(err, DUPLEX_DEVERR_NONFINITE);
    v = v > 0.f ? kFixClamp : (v < 0.f ? -kFixClamp : 0.f);
  }
  return (unsigned long long)__float2ll_rn(v * kFixScale);
}

// h = A (the fixed-point sum, [nT][H] int64) x 2^-32 (one rounding to fp32) (+ res, the
// previous MoE input in hpl), rounded once to T.  With `out` null every CTA converts all
// rows into its hpl (in place: each element is read and written by one thread), and a
// consumer barrier ends it; with `out` the CTA writes its share (CTA g of G takes every
// G-th group of 4 values) of the launch's result.
template <typename T>
DEVN void load_sum_rows(const unsigned long long* A, int nT, int H, bool residual, T* hpl,
                        T* out, int g, int G) {
  const int total = (nT * H) >> 2;  // groups of 4 values (32 bytes of A)
  const int first = out ? g * kConsumers + (int)threadIdx.x : (int)threadIdx.x;
  const int step = out ? G * kConsumers : kConsumers;
  for (int idx = first; idx < total; idx += step) {
    const longlong2* src = reinterpret_cast<const longlong2*>(A) + 2 * idx;
    const longlong2 a0 = __ldcg(src), a1 = __ldcg(src + 1);
    float v[4] = {__ll2float_rn(a0.x) * kFixInv, __ll2float_rn(a0.y) * kFixInv,
                  __ll2float_rn(a1.x) * kFixInv, __ll2float_rn(a1.y) * kFixInv};
    union {
      uint2 u;
      T h[4];
    } pk;
    if (residual) {
      pk.u = *reinterpret_cast<const uint2*>(hpl + (size_t)idx * 4);
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] += to_f32<T>(pk.h[k]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) pk.h[k] = from_f32<T>(v[k]);
    *reinterpret_cast<uint2*>((out ? out : hpl) + (size_t)idx * 4) = pk.u;
  }
  if (!out) named_bar_sync(1, kConsumers);
}

// The MoE layer input in one pass: h = A x 2^-32 (+ res, the previous MoE input in
// hpl), rounded once to T, into hpl; each warp's sums of squares of the rounded values
// per token (fixed order: the thread's groups in order, an xor butterfly, then the
// warps in order -- every thread adds the 16 warp sums itself, so all get the same
// bits without a second barrier) give the RMS scale; each thread then normalises its
// own groups into xsh (natural order).  Two consumer barriers.
template <typename T, int KT>
DEVN void input_rows(const unsigned long long* A, int nT, int H, bool residual, bool rms,
                     float eps, T* hpl, float* inv, uint8_t* xsh, uint32_t pitch, float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gpt = H >> 2;  // groups of 4 values per token
  const int total = nT * gpt;
  float ss[KT];
#pragma unroll
  for (int n = 0; n < KT; ++n) ss[n] = 0.f;
  for (int idx = tid; idx < total; idx += kConsumers) {
    const int n = idx / gpt;
    const longlong2* src = reinterpret_cast<const longlong2*>(A) + 2 * idx;
    const longlong2 a0 = __ldcg(src), a1 = __ldcg(src + 1);
    float v[4] = {__ll2float_rn(a0.x) * kFixInv, __ll2float_rn(a0.y) * kFixInv,
                  __ll2float_rn(a1.x) * kFixInv, __ll2float_rn(a1.y) * kFixInv};
    union {
      uint2 u;
      T h[4];
    } pk;
    if (residual) {
      pk.u = *reinterpret_cast<const uint2*>(hpl + (size_t)idx * 4);
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] += to_f32<T>(pk.h[k]);
    }
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      pk.h[k] = from_f32<T>(v[k]);
      const float r = to_f32<T>(pk.h[k]);
      sq = fmaf(r, r, sq);
    }
    *reinterpret_cast<uint2*>(hpl + (size_t)idx * 4) = pk.u;
    if (!rms)
      *reinterpret_cast<uint2*>(xsh + (uint32_t)n * pitch + (uint32_t)(idx - n * gpt) * 8u) = pk.u;
#pragma unroll
    for (int m = 0; m < KT; ++m)
      if (m == n) ss[m] += sq;
  }
  if (rms) {
#pragma unroll
    for (int n = 0; n < KT; ++n) {
      float a = ss[n];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && n < nT) scratch[warp * kMaxTokens + n] = a;
    }
    named_bar_sync(1, kConsumers);
    float sc[KT];
#pragma unroll
    for (int n = 0; n < KT; ++n) {
      float a = 0.f;
      if (n < nT) {
#pragma unroll
        for (int w = 0; w < kCW; ++w) a += scratch[w * kMaxTokens + n];
      }
      sc[n] = 1.0f / sqrtf(a / (float)H + eps);
      if (tid == n && n < nT) inv[n] = sc[n];
    }
    for (int idx = tid; idx < total; idx += kConsumers) {
      const int n = idx / gpt;
      float s = sc[0];
#pragma unroll
      for (int m = 1; m < KT; ++m)
        if (m == n) s = sc[m];
      union {
        uint2 u;
        T h[4];
      } pk;
      pk.u = *reinterpret_cast<const uint2*>(hpl + (size_t)idx * 4);
#pragma unroll
      for (int k = 0; k < 4; ++k) pk.h[k] = from_f32<T>(to_f32<T>(pk.h[k]) * s);
      *reinterpret_cast<uint2*>(xsh + (uint32_t)n * pitch + (uint32_t)(idx - n * gpt) * 8u) = pk.u;
    }
  }
  named_bar_sync(1, kConsumers);
}

// Zero CTA g's share (of G) of an accumulator of n int64 values (n % 2 == 0).
DEVI void zero_share(unsigned long long* A, int n, int g, int G) {
  const int pairs = n >> 1;
  for (int i = g * kConsumers + (int)threadIdx.x; i < pairs; i += G * kConsumers)
    reinterpret_cast<longlong2*>(A)[i] = make_longlong2(0, 0);
}

// RMS scale per token from the full rows in hpl ([nT][H], natural order), fixed
// order: warp n sums row n.
template <typename T>
DEVN void local_inv_rms(const T* hpl, int nT, int H, float eps, float* inv) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp < nT) {
    float a = 0.f;
    for (int q = lane; q < (H >> 3); q += 32) {
      const uint4 v = *reinterpret_cast<const uint4*>(hpl + (size_t)warp * H + q * 8);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) a = fmaf(to_f32<T>(e[k]), to_f32<T>(e[k]), a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) inv[warp] = 1.0f / sqrtf(a / (float)H + eps);
  }
  named_bar_sync(1, kConsumers);
}

// Rows of hpl ([nT][H]) into xsh in natural order, RMS-normalised with `inv` (one
// rounding to T) when rms.
template <typename T>
DEVN void normalise_rows(const T* hpl, int nT, int H, const float* inv, bool rms, uint8_t* xsh,
                         uint32_t pitch) {
  const int nq = H >> 3;
  for (int idx = threadIdx.x; idx < nT * nq; idx += kConsumers) {
    const int n = idx / nq, q = idx - n * nq;
    uint4 v = *reinterpret_cast<const uint4*>(hpl + (size_t)n * H + q * 8);
    if (rms) {
      const float sc = inv[n];
      T* e = reinterpret_cast<T*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = from_f32<T>(to_f32<T>(e[k]) * sc);
    }
    *reinterpret_cast<uint4*>(xsh + (uint32_t)n * pitch + (uint32_t)q * 16u) = v;
  }
  named_bar_sync(1, kConsumers);
}

// Rows of a global [nT][H] buffer (written by other CTAs: read through L2) into hpl.
template <typename T>
DEVN void load_rows(const T* src, int nT, int H, T* hpl) {
  const int total = nT * (H >> 3);
  for (int idx = threadIdx.x; idx < total; idx += kConsumers)
    *reinterpret_cast<uint4*>(hpl + (size_t)idx * 8) =
        __ldcg(reinterpret_cast<const uint4*>(src + (size_t)idx * 8));
  named_bar_sync(1, kConsumers);
}

// ------------------------------------------------------------------ router
// Gate records (duplex_repack_gate_records): the gate matrix [E][H] in blocks of 16
// experts, per 16-column k-step the mma.sync A fragments of the 32 lanes (lane (g, t):
// rows g, g + 8 x columns 2t, 2t + 1, 2t + 8, 2t + 9), 512 bytes per (block, k-step).
// CTA `rank` of a cluster takes blocks rank, rank + 8, ...; a block's k-steps arrive in
// ring stages of `kps` k-steps.  Warp w takes k-steps [w KS / 16, (w + 1) KS / 16) of
// every block (B = the normalised tokens, natural order in xsh), the partial sums
// are added in warp order, and each logit, rounded to T (+ bias), goes to every CTA
// of the cluster: ls[n][e].  Every warp then releases every gate stage.
template <typename T>
DEVI void router_mma(const uint8_t* ring, uint32_t slot_bytes, int NS, RingPos pos, int rank,
                     int nblk, int KS, int kps, int E, int nT, const uint8_t* xsh, uint32_t pitch,
                     const void* gate_b, float* ls, float* red, uint64_t* full, uint64_t* empty,
                     volatile int* abort, int* err, long long limit) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool xon = g < nT;
  const int ks0 = (warp * KS) / kCW, ks1 = ((warp + 1) * KS) / kCW;
  const uint8_t* xrow = xsh + (uint32_t)g * pitch + (uint32_t)t * 4u;
  RingPos rp = pos;
  int nst = 0;
  for (int b = rank; b < nblk; b += kCS) {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < KS; k0 += kps, rp.next(NS), ++nst) {
      const int lo = ks0 > k0 ? ks0 : k0;
      const int hi = ks1 < k0 + kps ? ks1 : k0 + kps;
      if (lo >= hi) continue;
      wait_phase(&full[rp.slot], rp.phase, abort, err, kSiteFull, limit);
      const uint8_t* ap = ring + (uint32_t)rp.slot * slot_bytes + (uint32_t)(lo - k0) * 512u +
                          (uint32_t)lane * 16u;
      const uint8_t* xp = xrow + (uint32_t)lo * 32u;
      for (int ks = lo; ks < hi; ++ks, ap += 512, xp += 32) {
        const uint4 a = *reinterpret_cast<const uint4*>(ap);
        uint32_t b0 = 0u, b1 = 0u;
        if (xon) {
          b0 = *reinterpret_cast<const uint32_t*>(xp);
          b1 = *reinterpret_cast<const uint32_t*>(xp + 16);
        }
        MmaOp<T>::run(d, a.x, a.y, a.z, a.w, b0, b1);
      }
    }
    // partials [warp][token][row]; tokens 2t, 2t + 1 of rows g, g + 8
    float* rb = red + warp * 128;
    if (2 * t < nT) {
      rb[(2 * t) * 16 + g] = d[0];
      rb[(2 * t) * 16 + g + 8] = d[2];
    }
    if (2 * t + 1 < nT) {
      rb[(2 * t + 1) * 16 + g] = d[1];
      rb[(2 * t + 1) * 16 + g + 8] = d[3];
    }
    named_bar_sync(1, kConsumers);
    if (tid < nT * 16) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) a += red[w * 128 + tid];
      const int n = tid >> 4, e = b * 16 + (tid & 15);
      if (e < E) {
        if (gate_b) a += to_f32<T>(reinterpret_cast<const T*>(gate_b)[e]);
        a = to_f32<T>(from_f32<T>(a));
#pragma unroll
        for (int q = 0; q < kCS; ++q) st_peer_f32(peer_addr(ls + n * E + e, (uint32_t)q), a);
      }
    }
    named_bar_sync(1, kConsumers);
  }
  __syncwarp();
  if (lane == 0) {
    RingPos r = pos;
    for (int j = 0; j < nst; ++j, r.next(NS)) mbar_arrive(&empty[r.slot]);
  }
}

// ------------------------------------------------------------------ routing plan
// plan_units for one token: warp 0 alone (lane holds experts lane + 32 i), the same
// keys and max-reductions as the general path, so the same selection; the units are
// the k selected experts in ascending id order (position = number of selected ids
// below).  With norm it also writes the renormalised routing weights.  A function of
// its own: inside plan_units the general path's code made this path ~2.5x slower
// (3,100 vs 1,250 cycles measured).
template <typename T, int KPL>  // KPL: keys per lane, E <= 32 KPL
DEVN int plan_one(int E, int top_k, int norm, uint8_t* smem, float* scratch, uint64_t* ready) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* ls = reinterpret_cast<const float*>(smem + kSLogit);
  int* sel_s = reinterpret_cast<int*>(smem + kSSel);
  int* unit_e = reinterpret_cast<int*>(smem + kSUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kSUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);
  int* n_units_s = reinterpret_cast<int*>(smem + kSNUnits);
  int* unit_of =  // plan_units's layout of the scratch, read again by plan_weights
      reinterpret_cast<int*>(scratch) + kMaxTokens * kMaxExperts + kMaxTokens * (kMaxExperts / 4);
  (void)tid;
  if (warp == 0) {
    uint32_t key[KPL];
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      const int e = lane + 32 * i;
      key[i] = e < E ? order_key<T>(ls[e], e) : 0u;
    }
    int sel[kMaxTopK];
    int mine = 0;  // lane j's pick
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      sel[j] = 0;
      if (j < top_k) {
        uint32_t lm = 0u;
#pragma unroll
        for (int i = 0; i < KPL; ++i) lm = key[i] > lm ? key[i] : lm;
        const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
#pragma unroll
        for (int i = 0; i < KPL; ++i)
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
    // renormalised top-k weights: the softmax denominator over all experts cancels,
    // so p_j / sum_i p_i = exp(l_j - l_max) / sum over the selection (in order)
    const float lmax = ls[sel[0]];
    const float ej = lane < top_k ? expf(ls[mine] - lmax) : 0.f;
    float esum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      const float x = __shfl_sync(0xffffffffu, ej, j);
      if (j < top_k) esum += x;
    }
    if (lane < top_k) {
      sel_s[lane] = mine;
      unit_of[mine] = rank;
      unit_e[rank] = mine;
      unit_m[rank] = 1u;
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) unit_w[rank * kMaxTokens + n] = 0.f;
      if (norm) unit_w[rank * kMaxTokens] = ej / esum;
    }
    if (lane == 0) *n_units_s = top_k;
    // the producer needs only the unit list: release it now, not after the barrier
    __syncwarp();
    if (lane == 0) mbar_arrive(ready);
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
DEVN int plan_units(int nT, int E, int top_k, uint8_t* smem, float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* ls = reinterpret_cast<const float*>(smem + kSLogit);
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
    const int tk = idx / E;
    keys[idx] = order_key<T>(ls[idx], idx - tk * E);
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

// ------------------------------------------------------------------ items
// A CTA takes its items in batches of up to p.ib: the gate|up tile pairs of the
// batch (partial sums of each warp deferred in `red`), one pass of sums, one
// exchange of the batch's intermediate rows, then the down records, two items per
// ring stage.


// Gate (x) and up (y) sums of output o = jj * nT * 16 + token * 16 + row, warps in order.
DEVI float2 sum_pair_partials(const float* red, int o, int nT) {
  const int per = nT * 16;
  const int jj = o / per, rem = o - jj * per;
  float v = 0.f, v2 = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) {
    v += red[((jj * 2) * kCW + w) * per + rem];
    v2 += red[((jj * 2 + 1) * kCW + w) * per + rem];
  }
  return make_float2(v, v2);
}

// After the batch's gate|up partials are in `red`: SiLU(gate) * up of this CTA's 16
// rows for each (item, token) (0 for tokens outside the item's unit), rounded to T,
// in fragment order (fp16: odd columns / 16) into rows [16 rank, 16 rank + 16) of xd
// (row item * nT + token) of every CTA of the cluster, with the partial column sums
// of those stored values (even, odd columns, as stage_rows sums them) into
// dgp[item][rank][token] of every CTA; then one arrival on every CTA's `bar`.  Thread
// o < nbt * nT * 16 holds row o & 15 of (item, token) o >> 4; an 8-lane group gathers
// its 8 rows by shuffles and lane j of the group writes CTA j.
template <typename T>
DEVI void act_send(const float* red, int nbt, int nT, int b0, int S, const uint32_t* unit_m,
                   int rank, uint8_t* xd, float2* dgp, uint64_t* bar) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int total = nbt * nT * 16;
  if ((tid & ~31) < total) {  // whole warps: every lane takes part in the shuffles
    const bool on = tid < total;
    float x = 0.f;
    int k = 0, n = 0;
    if (on) {
      const float2 v = sum_pair_partials(red, tid, nT);
      k = tid / (nT * 16);
      n = (tid >> 4) - k * nT;
      const int u = (b0 + k) / S;
      x = ((unit_m[u] >> n) & 1u) ? silu_f32(v.x) * v.y : 0.f;
    }
    x = to_f32<T>(from_f32<T>(x));
    const int base = lane & ~7, j = lane & 7;
    union {
      uint4 u;
      T h[8];
    } pk;
#pragma unroll
    for (int q = 0; q < 8; ++q) pk.h[q] = from_f32<T>(__shfl_sync(0xffffffffu, x, base + q));
    uint4 o = to_frag_order(pk.u);
    if (DqOff<T>::kOddDiv16) {
      const __half2 q16 = __float2half2_rn(0.0625f);
      __half2 hy = __hmul2(*reinterpret_cast<__half2*>(&o.y), q16);
      __half2 hw = __hmul2(*reinterpret_cast<__half2*>(&o.w), q16);
      o.y = *reinterpret_cast<uint32_t*>(&hy);
      o.w = *reinterpret_cast<uint32_t*>(&hw);
    }
    const T* e = reinterpret_cast<const T*>(&o);
    float se = (to_f32<T>(e[0]) + to_f32<T>(e[1])) + (to_f32<T>(e[4]) + to_f32<T>(e[5]));
    float so = (to_f32<T>(e[2]) + to_f32<T>(e[3])) + (to_f32<T>(e[6]) + to_f32<T>(e[7]));
    se += __shfl_xor_sync(0xffffffffu, se, 8);  // the other half of the 16 rows
    so += __shfl_xor_sync(0xffffffffu, so, 8);
    if (on) {
      const int h = (tid >> 3) & 1, r = k * nT + n;
      st_peer_v4(peer_addr(xd + (uint32_t)r * kXdPitch + (uint32_t)(rank * 16 + h * 8) * 2u,
                           (uint32_t)j),
                 o);
      if (h == 0)
        st_peer_v2(peer_addr(dgp + (k * kCS + rank) * 8 + n, (uint32_t)j),
                   make_uint2(__float_as_uint(se), __float_as_uint(so)));
    }
  }
  signal_cluster_xchg(bar);
}

// (P, Q) of the offset path from column sums (se: even columns, so: odd, as stored).
template <typename T>
DEVI float2 corr_pq(float se, float so) {
  if (DqOff<T>::kOddDiv16) return make_float2(1024.f * (se + so), fmaf(16.f, so, se));
  const float q = se + so;
  return make_float2(128.f * q, q);
}

// Correction sums of the staged slices per window of 32 columns (`cw` = 1, group 32)
// or pair of 64 (`cw` = 2) from the CTAs' partials, dg [item][window][8 tokens]
// (the general path; the group-128 path adds the partials inside the down loop).
template <typename T>
DEVI void dg_from_partials(const float2* dgp, int nbt, int nT, int cw, float2* dg) {
  const int tid = threadIdx.x;
  const int nwin = kSliceK / (32 * cw), per = kCS / nwin;
  if (tid < nbt * nT * nwin) {
    const int wi = tid % nwin, r = tid / nwin;
    const int k = r / nT, n = r - k * nT;
    float se = 0.f, so = 0.f;
    for (int q = wi * per; q < (wi + 1) * per; ++q) {
      const float2 v = dgp[(k * kCS + q) * 8 + n];
      se += v.x;
      so += v.y;
    }
    dg[(k * nwin + wi) * 8 + n] = corr_pq<T>(se, so);
  }
  named_bar_sync(1, kConsumers);
}

// One K-slice record (16 output rows x 128 columns, group 128: one group of two
// pairs) against the staged slice rows xd (token g of lane (g, t)): acc += w * dot.
template <typename T, typename S>
DEVI void ks_record_g128(const uint8_t* rec, const TileGeom& tg, int lane, const uint8_t* xd,
                         const float2* dgp, float w0, float w1, bool xon, float (&acc)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* xrow = xd + (uint32_t)g * kXdPitch + (uint32_t)t * 16u;
  const uint8_t* wp = rec + (uint32_t)lane * 16u;
  // the slice's column sums for tokens 2t, 2t + 1: the 8 CTAs' partials in rank order
  float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < kCS; ++q) {
    const float4 v = *reinterpret_cast<const float4*>(dgp + q * 8 + 2 * t);
    c.x += v.x;
    c.y += v.y;
    c.z += v.z;
    c.w += v.w;
  }
  const float2 pq0 = corr_pq<T>(c.x, c.y), pq1 = corr_pq<T>(c.z, c.w);
  const float4 gs = make_float4(pq0.x, pq0.y, pq1.x, pq1.y);
  float d[4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
    if (xon) {
      xa = *reinterpret_cast<const uint4*>(xrow + k * 128);
      xb = *reinterpret_cast<const uint4*>(xrow + k * 128 + 64);
    }
    const uint4 w = *reinterpret_cast<const uint4*>(wp + k * 512);
    uint32_t A[4], B[4];
    DqOff<T>::expand(w.x, w.y, A, B);
    if (k == 0)
      mma_first<T>(d, A[0], A[1], A[2], A[3], xa.x, xa.y);
    else
      MmaOp<T>::run(d, A[0], A[1], A[2], A[3], xa.x, xa.y);
    MmaOp<T>::run(d, B[0], B[1], B[2], B[3], xa.z, xa.w);
    DqOff<T>::expand(w.z, w.w, A, B);
    MmaOp<T>::run(d, A[0], A[1], A[2], A[3], xb.x, xb.y);
    MmaOp<T>::run(d, B[0], B[1], B[2], B[3], xb.z, xb.w);
  }
  const float zero4v[4] = {0.f, 0.f, 0.f, 0.f};
  flush_group<S>(acc, d, zero4v, rec, tg, 0, g, gs, w0, w1);
}

// Down projection of `nit` (1 or 2) items of a DN stage (item j's records at st + j *
// dn_bytes) for this warp's records (16 output rows each): K = the item's 128-column
// slice in xd (rows j * nT + token), weights w[j] of its unit's tokens.
template <typename T, typename S, bool G32>
DEVI void slice_down(const uint8_t* st, const TileGeom tg, int nrec, uint32_t dn_bytes, int nit,
                     const uint8_t* xd, const float2* dgp, const float2* dg, int nwin,
                     const float* w0, const float* w1, int nT, float (&acc)[kMaxRecPerWarp][4],
                     uint64_t* empty_bar) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool xon = (lane >> 2) < nT;
  const int t = lane & 3;
  for (int j = 0; j < nit; ++j) {
    const float* w = j ? w1 : w0;
#pragma unroll
    for (int k = 0; k < kMaxRecPerWarp; ++k) {
      const int rec = warp + k * kCW;
      if (rec >= nrec) continue;
      const uint8_t* r = st + j * dn_bytes + (uint32_t)rec * tg.rec_bytes;
      const uint8_t* xj = xd + (uint32_t)(j * nT) * kXdPitch;
      if (!G32 && tg.gshift == 1)
        ks_record_g128<T, S>(r, tg, lane, xj, dgp + j * kCS * 8, w[2 * t], w[2 * t + 1], xon,
                             acc[k]);
      else
        rm_offset<T, S, G32>(r, tg, 0, tg.npairs, lane, xj, kXdPitch, 0, dg + j * nwin * 8, 0, w,
                             xon, acc[k]);
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);
}

// This CTA's rows of the cluster's partial output: part[c][n][row] (fp32).
// This CTA's partial output rows (the down projection's accumulators, warp w holding
// records w, w + 16) added into the fixed-point accumulator A ([nT][H]).
DEVI void add_partials(unsigned long long* A, int nT, int H, int row0, int nrec,
                       float (&acc)[kMaxRecPerWarp][4], int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k = 0; k < kMaxRecPerWarp; ++k) {
    const int rec = warp + k * kCW;
    if (rec < nrec) {
      const int row = row0 + rec * 16 + g;
      if (2 * t < nT) {
        atomicAdd(A + (size_t)(2 * t) * H + row, to_fix(acc[k][0], err));
        atomicAdd(A + (size_t)(2 * t) * H + row + 8, to_fix(acc[k][2], err));
      }
      if (2 * t + 1 < nT) {
        atomicAdd(A + (size_t)(2 * t + 1) * H + row, to_fix(acc[k][1], err));
        atomicAdd(A + (size_t)(2 * t + 1) * H + row + 8, to_fix(acc[k][3], err));
      }
    }
    zero4(acc[k]);
  }
}

DEVI void item_range(int n_items, int C, int c, int& i0, int& i1) {
  i0 = (int)((long long)n_items * c / C);
  i1 = (int)((long long)n_items * (c + 1) / C);
}

// NT: 1 for the one-token kernel (the per-token loops fold away), 0 for T from p.T.
template <typename T, typename S, bool G32, int NT>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(const __grid_constant__ StackParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kSEmpty);
  uint64_t* plan_ready = reinterpret_cast<uint64_t*>(smem + kSPlan);
  uint64_t* lg_full = reinterpret_cast<uint64_t*>(smem + kSLg);
  uint64_t* act_full = reinterpret_cast<uint64_t*>(smem + kSAct);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSAbort);
  int* n_units_s = reinterpret_cast<int*>(smem + kSNUnits);
  int* unit_e = reinterpret_cast<int*>(smem + kSUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kSUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kSUnitW);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nslots;
  const int cta = blockIdx.x, G = gridDim.x;
  const int rank = (int)cluster_ctarank();
  const int cid = (int)cluster_id_x();
  const int C = (int)nclusters_x();
  const long long limit = p.wait_limit;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], kCW);
    }
    mbar_init(plan_ready, 1);
    mbar_init(lg_full, kCS);
    mbar_init(&act_full[0], kCS);
    mbar_init(&act_full[1], kCS);
    // an earlier launch that gave up leaves the bit set: give up at once
    *abort_flag = (*reinterpret_cast<volatile int*>(p.err) & DUPLEX_DEVERR_TIMEOUT) ? 1 : 0;
    fence_mbar_init();
  }
  // every CTA's barriers exist before any CTA of the cluster arrives on them
  cluster_sync_all();

  const int perG = p.I >> 4;             // gate|up tiles per unit
  const int spb = (p.KS + p.kps - 1) / p.kps;                   // ring stages per gate block
  const int ngs = (p.nblk > rank ? (p.nblk - rank + kCS - 1) / kCS : 0) * spb;  // per layer
  const int nrec = p.rrows >> 4;             // down records of this CTA per item
  const int row0 = rank * p.rrows;

  if (warp == kCW) {
    // ================================================================ producer
    if (lane == 0) {
      // the producer waits on the consumers: a longer limit, so that a stuck consumer
      // wait is the one that gives up (and names its site)
      const long long plimit = 4 * limit;
      const uint64_t pol = policy_evict_first();
      int i = 0;  // stage sequence number
      RingPos wp = {0, 0u};
      bool ok = true;
      // one stage of one or two copies of `bytes` each, side by side in the slot; weights
      // read once carry the evict-first hint, the gate records (read by every cluster)
      // stay in L2 for the other clusters
      auto issue2 = [&](const uint8_t* src0, const uint8_t* src1, uint32_t bytes,
                        bool keep = false) {
        if (i >= NS)  // the slot's previous stage has been released by every consumer warp
          wait_phase(&empty[wp.slot], wp.phase ^ 1u, abort_flag, p.err, kSiteEmpty, plimit);
        if (*abort_flag) {
          ok = false;
          return;
        }
        uint8_t* dst = smem + p.off_ring + (uint32_t)wp.slot * p.slot_bytes;
        mbar_arrive_expect_tx(&full[wp.slot], src1 ? 2u * bytes : bytes);
        if (keep)
          bulk_g2s(dst, src0, bytes, &full[wp.slot]);
        else
          bulk_g2s_stream(dst, src0, bytes, &full[wp.slot], pol);
        if (src1) bulk_g2s_stream(dst + bytes, src1, bytes, &full[wp.slot], pol);
        mbar_arrive(&full[wp.slot]);
        ++i;
        wp.next(NS);
      };
      auto issue = [&](const uint8_t* src, uint32_t bytes, bool keep = false) {
        issue2(src, nullptr, bytes, keep);
      };
      for (int l = 0; l < p.n_layers && ok; ++l) {
        const duplex_stack_layer L = p.layers[l];
        if (p.has_attn) {
          for (int t = cta; t < p.RbQ && ok; t += G)
            issue(reinterpret_cast<const uint8_t*>(L.qkv_tiles) + (size_t)t * p.tq.rec_bytes,
                  p.tq.rec_bytes);
          for (int t = cta; t < p.RbO && ok; t += G)
            issue(reinterpret_cast<const uint8_t*>(L.o_tiles) + (size_t)t * p.to.rec_bytes,
                  p.to.rec_bytes);
        }
        for (int b = rank; b < p.nblk && ok; b += kCS)
          for (int k = 0; k < spb && ok; ++k) {
            const int nks = (p.KS - k * p.kps) < p.kps ? (p.KS - k * p.kps) : p.kps;
            issue(reinterpret_cast<const uint8_t*>(L.gate_w) +
                      ((size_t)b * p.KS + (size_t)k * p.kps) * 512u,
                  (uint32_t)nks * 512u, true);
          }
        if (!ok) break;
        // routing plan of this layer (built by this CTA's consumers)
        wait_phase(plan_ready, (uint32_t)(l & 1), abort_flag, p.err, kSitePlan, plimit);
        if (*abort_flag) break;
        int nu = *n_units_s;
        nu = nu < 0 ? 0 : (nu > kMaxUnits ? kMaxUnits : nu);
        int i0, i1;
        item_range(nu * p.S, C, cid, i0, i1);
        auto expert = [&](int it) {
          int e = unit_e[it / p.S];
          if ((unsigned)e >= (unsigned)p.E) {  // never turn a bad id into an address
            set_error(p.err, DUPLEX_DEVERR_EXPERT);
            e = 0;
          }
          return e;
        };
        auto dn_src = [&](int it) {
          return reinterpret_cast<const uint8_t*>(L.dn_tiles) +
                 (((size_t)expert(it) * p.S + it % p.S) * (p.H >> 4) + (size_t)rank * nrec) *
                     p.tks.rec_bytes;
        };
        for (int b0 = i0; b0 < i1 && ok; b0 += p.ib) {
          const int nbt = (i1 - b0) < p.ib ? (i1 - b0) : p.ib;
          for (int k = 0; k < nbt && ok; ++k) {
            const int it = b0 + k;
            issue(reinterpret_cast<const uint8_t*>(L.gu_tiles) +
                      ((size_t)expert(it) * (2 * perG) + 2 * ((it % p.S) * kCS + rank)) *
                          p.tgu.rec_bytes,
                  2u * p.tgu.rec_bytes);
          }
          for (int k = 0; k < nbt && ok; k += 2) {
            if (k + 1 < nbt)
              issue2(dn_src(b0 + k), dn_src(b0 + k + 1), p.dn_bytes);
            else
              issue(dn_src(b0 + k), p.dn_bytes);
          }
        }
      }
      // drain: never leave the CTA while a bulk copy may still target its smem
      const int first = i > NS ? i - NS : 0;
      for (int j = first; j < i; ++j) {
        const long long t0 = clock64();
        bool done = true;
        while (!mbar_try_wait(&full[j % NS], (uint32_t)(j / NS) & 1u))
          if (clock64() - t0 > 200000000LL) {
            done = false;
            break;
          }
        if (!done) {
          give_up(abort_flag, p.err, kSiteDrain);
          break;
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // no CTA leaves while a peer may still write into its smem
    return;
  }

  // ================================================================== consumers
  float* red = reinterpret_cast<float*>(smem + kSRed);
  float* ls = reinterpret_cast<float*>(smem + kSLogit);
  float* inv = reinterpret_cast<float*>(smem + kSInv);
  float2* dgp0 = reinterpret_cast<float2*>(smem + p.off_av);  // [2][ib][kCS][8] partial sums
  float2* dg = reinterpret_cast<float2*>(smem + p.off_dg);
  const int nwin = kSliceK / (32 * (G32 ? 1 : 2));
  uint8_t* xsh = smem + p.off_x;
  float2* gsum = reinterpret_cast<float2*>(smem + p.off_gsum);
  T* hpl = reinterpret_cast<T*>(smem + p.off_h);
  const int nT = NT ? NT : p.T;
  constexpr int KT = NT ? NT : kMaxTokens;
  const int cw = G32 ? 1 : 2;
  const bool rms = p.rms_eps > 0.f;
  int* err = p.err;
  int i = 0;        // stage sequence number
  unsigned nb = 0;  // grid barriers passed
  int kbatch = 0;   // item batches done (intermediate buffer parity)
  float acc[kMaxRecPerWarp][4];
#pragma unroll
  for (int k = 0; k < kMaxRecPerWarp; ++k) zero4(acc[k]);

  RingPos rp = {0, 0u};  // the consumers' position in the ring (stage i)
  auto wait_full = [&]() { wait_phase(&full[rp.slot], rp.phase, abort_flag, err, kSiteFull, limit); };
  auto slot_ptr = [&]() { return smem + p.off_ring + (uint32_t)rp.slot * p.slot_bytes; };
  auto next_stage = [&]() {
    ++i;
    rp.next(NS);
  };
  auto sync_grid = [&]() {
    grid_arrive(p.barrier);
    ++nb;
    grid_wait(p.barrier, nb, nb == 1 && (p.test_flags & 1), abort_flag, err, limit);
  };
  auto accbuf = [&](int l) { return p.acc + (size_t)(l % 3) * nT * p.H; };

  for (int l = 0; l < p.n_layers; ++l) {
    const duplex_stack_layer L = p.layers[l];
    // ------------------------------------------------------------------ h
    if (l == 0) {
      load_rows<T>(reinterpret_cast<const T*>(p.x_in), nT, p.H, hpl);
      if (rms) local_inv_rms<T>(hpl, nT, p.H, p.rms_eps, inv);
      normalise_rows<T>(hpl, nT, p.H, inv, rms, xsh, p.x_pitch);
    } else {
      ++nb;
      grid_wait(p.barrier, nb, nb == 1 && (p.test_flags & 1), abort_flag, err, limit);
      input_rows<T, KT>(accbuf(l - 1), nT, p.H, p.moe_residual != 0, rms, p.rms_eps, hpl, inv,
                        xsh, p.x_pitch, red);
    }
    // the accumulator of layer l + 1 was last read at the start of layer l - 1, and is
    // next added into after this layer's grid barrier
    zero_share(accbuf(l + 1), nT * p.H, cta, G);
    if (p.has_attn) {
      // -------------------------------------------------------------- Q
      stage_rows<T>(nullptr, 0, nT, p.H, xsh, p.x_pitch, gsum, cw, kStageFrag);
      {
        const int rmax = defer_tiles(nT);
        int j = 0, t0 = cta;
        for (int tile = cta; tile < p.RbQ; tile += G, next_stage()) {
          wait_full();
          tile_acc<T, S, 1, G32>(slot_ptr(), p.tq, xsh, p.x_pitch, gsum, nT, &empty[rp.slot], red,
                                 j++);
          if (j == rmax || tile + G >= p.RbQ) {
            named_bar_sync(1, kConsumers);
            if (tid < j * nT * 16) {
              const float v = sum_partials(red, tid, nT);
              const int jj = tid / (nT * 16), n = (tid >> 4) - jj * nT;
              const int row = (t0 + jj * G) * 16 + (tid & 15);
              if (row < p.qkv_R)
                reinterpret_cast<T*>(p.qkv)[(size_t)n * p.qkv_R + row] = from_f32<T>(v);
            }
            named_bar_sync(1, kConsumers);
            j = 0;
            t0 = tile + G;
          }
        }
      }
      sync_grid();
      // -------------------------------------------------------------- O
      if (cta < p.RbO)
        stage_rows<T>(reinterpret_cast<const uint8_t*>(p.qkv), p.qkv_R, nT, p.q_dim, xsh,
                      p.x_pitch, gsum, cw, kStageAll);
      {
        const int rmax = defer_tiles(nT);
        int j = 0, t0 = cta;
        for (int tile = cta; tile < p.RbO; tile += G, next_stage()) {
          wait_full();
          tile_acc<T, S, 1, G32>(slot_ptr(), p.to, xsh, p.x_pitch, gsum, nT, &empty[rp.slot], red,
                                 j++);
          if (j == rmax || tile + G >= p.RbO) {
            named_bar_sync(1, kConsumers);
            if (tid < j * nT * 16) {
              const float v = sum_partials(red, tid, nT);
              const int jj = tid / (nT * 16), n = (tid >> 4) - jj * nT;
              const int row = (t0 + jj * G) * 16 + (tid & 15);
              if (row < p.H) {
                const float res = to_f32<T>(hpl[(size_t)n * p.H + row]);
                reinterpret_cast<T*>(p.h1)[(size_t)n * p.H + row] =
                    from_f32<T>(to_f32<T>(from_f32<T>(v)) + res);
              }
            }
            named_bar_sync(1, kConsumers);
            j = 0;
            t0 = tile + G;
          }
        }
      }
      sync_grid();
      // the MoE input (and residual): h1 from every CTA's o rows
      load_rows<T>(reinterpret_cast<const T*>(p.h1), nT, p.H, hpl);
      if (rms) local_inv_rms<T>(hpl, nT, p.H, p.rms_eps, inv);
      normalise_rows<T>(hpl, nT, p.H, inv, rms, xsh, p.x_pitch);
    }
    // ------------------------------------------------------------------ router
    router_mma<T>(smem + p.off_ring, p.slot_bytes, NS, rp, rank, p.nblk, p.KS, p.kps, p.E, nT,
                  xsh, p.x_pitch, L.gate_b, ls, red, full, empty, abort_flag, err, limit);
    for (int k = 0; k < ngs; ++k) next_stage();
    signal_cluster_xchg(lg_full);
    // fragment-order staging of the normalised tokens while the logits travel
    stage_rows<T>(nullptr, 0, nT, p.H, xsh, p.x_pitch, gsum, cw, kStageFrag);
    wait_cluster_xchg(lg_full, (uint32_t)(l & 1), abort_flag, err, limit);
    // ------------------------------------------------------------------ plan
    const int nu = nT != 1   ? plan_units<T>(nT, p.E, p.top_k, smem, red)
                   : p.E <= 128 ? plan_one<T, 4>(p.E, p.top_k, p.norm, smem, red, plan_ready)
                                : plan_one<T, kMaxExperts / 32>(p.E, p.top_k, p.norm, smem, red,
                                                                plan_ready);
    if (nT != 1 && tid == 0) mbar_arrive(plan_ready);
    if (nT != 1 || !p.norm) plan_weights(nT, p.E, p.top_k, p.norm, smem, red);
    // ------------------------------------------------------------------ items
    int i0, i1;
    item_range(nu * p.S, C, cid, i0, i1);
    for (int b0 = i0; b0 < i1; b0 += p.ib) {
      const int nbt = (i1 - b0) < p.ib ? (i1 - b0) : p.ib;
      const int b = kbatch & 1;
      uint8_t* xd = smem + p.off_xd + (uint32_t)b * (uint32_t)(p.ib * nT) * kXdPitch;
      // gate|up tile pairs (slice rows [16 rank, 16 rank + 16)), partials deferred
      for (int k = 0; k < nbt; ++k, next_stage()) {
        wait_full();
        tile_acc<T, S, 2, G32>(slot_ptr(), p.tgu, xsh, p.x_pitch, gsum, nT, &empty[rp.slot], red,
                               k);
      }
      named_bar_sync(1, kConsumers);
      float2* dgp = dgp0 + (uint32_t)b * (uint32_t)(p.ib * kCS * 8);
      act_send<T>(red, nbt, nT, b0, p.S, unit_m, rank, xd, dgp, &act_full[b]);
      wait_cluster_xchg(&act_full[b], (uint32_t)((kbatch >> 1) & 1), abort_flag, err, limit);
      if (G32 || p.tks.gshift != 1) dg_from_partials<T>(dgp, nbt, nT, cw, dg);
      // down: this CTA's output rows x each item's 128 columns, two items per stage
      for (int k = 0; k < nbt; k += 2, next_stage()) {
        const int nit = (nbt - k) < 2 ? 1 : 2;
        const int u0 = (b0 + k) / p.S, u1 = (b0 + k + nit - 1) / p.S;
        wait_full();
        slice_down<T, S, G32>(slot_ptr(), p.tks, nrec, p.dn_bytes, nit,
                              xd + (uint32_t)(k * nT) * kXdPitch, dgp + k * kCS * 8,
                              dg + k * nwin * 8, nwin,
                              unit_w + u0 * kMaxTokens, unit_w + u1 * kMaxTokens, nT, acc,
                              &empty[rp.slot]);
      }
      ++kbatch;
    }
    // ------------------------------------------------------------------ end of layer
    add_partials(accbuf(l), nT, p.H, row0, nrec, acc, err);
    grid_arrive(p.barrier);
  }
  // the result: every CTA converts its share of the last layer's sum
  ++nb;
  grid_wait(p.barrier, nb, nb == 1 && (p.test_flags & 1), abort_flag, err, limit);
  load_sum_rows<T>(accbuf(p.n_layers - 1), nT, p.H, p.moe_residual != 0, hpl,
                   reinterpret_cast<T*>(p.out), cta, G);
  cluster_sync_all();
}

// ---------------------------------------------------------------- down K-slices
// Record (e, s, rb): rows [16 rb, 16 rb + 16) x columns [128 s, 128 s + 128) of
// expert e's down matrix [H][I] in the tile-record layout of tiles.cuh (K = 128, its
// 128 / group groups), padded to 16 bytes; records ordered [E][I / 128][H / 16].
template <typename S>
__global__ void slice_repack_kernel(const int32_t* __restrict__ packed,
                                    const S* __restrict__ scale, const int32_t* __restrict__ zeros,
                                    int E, int H, int I, int G, int GZ, TileGeom tg,
                                    uint32_t* __restrict__ out) {
  const int Rb = H >> 4, NSl = I / kSliceK, C = I >> 3;
  const uint32_t wpr = tg.rec_bytes / 4u;
  const long long total = (long long)E * NSl * Rb * wpr;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long rec = idx / wpr;
    const uint32_t o = (uint32_t)(idx - rec * wpr) * 4u;
    const int rb = (int)(rec % Rb);
    const long long es = rec / Rb;
    const int s = (int)(es % NSl), e = (int)(es / NSl);
    uint32_t val = 0;
    if (o < tg.off_scale) {
      const int pr = (int)(o >> 9);
      const int ln = (int)((o & 511u) >> 4);
      const int j = (int)((o & 15u) >> 2);
      const int g = ln >> 2, t = ln & 3;
      const int row = rb * 16 + g + ((j & 1) ? 8 : 0);
      const int word = s * (kSliceK / 8) + 8 * pr + t + ((j & 2) ? 4 : 0);
      val = (uint32_t)packed[((long long)e * H + row) * C + word];
    } else if (o < tg.off_zero) {
      const int q = (int)((o - tg.off_scale) >> 2);
      const int grp = s * tg.Gr + (q >> 3), g = q & 7;
      const int ra = rb * 16 + g, rbw = ra + 8;
      const uint16_t sa = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * H + ra) * G + grp]);
      const uint16_t sb = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * H + rbw) * G + grp]);
      val = (uint32_t)sa | ((uint32_t)sb << 16);
    } else if (tg.has_zeros && o < tg.off_zero + (uint32_t)tg.Gr * 8u) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int q = (int)(o - tg.off_zero) + b;
        const int grp = s * tg.Gr + (q >> 3), g = q & 7;
        const int ra = rb * 16 + g, rbw = ra + 8;
        const uint32_t za =
            ((uint32_t)zeros[((long long)e * H + ra) * GZ + (grp >> 3)] >> ((grp & 7) * 4)) & 15u;
        const uint32_t zb =
            ((uint32_t)zeros[((long long)e * H + rbw) * GZ + (grp >> 3)] >> ((grp & 7) * 4)) & 15u;
        val |= (za | (zb << 4)) << (8 * b);
      }
    }
    out[idx] = val;
  }
}

// Gate records: word j of lane (g, t) for (block b, k-step ks) is the mma.sync A
// register j of rows 16 b + g (j = 0, 2) or 16 b + g + 8 (j = 1, 3), columns
// 16 ks + 2t, 2t + 1 (j = 0, 1) or 16 ks + 2t + 8, 2t + 9 (j = 2, 3); rows past E are 0.
__global__ void gate_repack_kernel(const uint16_t* __restrict__ w, int E, int H,
                                   uint32_t* __restrict__ out) {
  const int KS = H >> 4;
  const long long total = (long long)((E + 15) >> 4) * KS * 128;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(idx & 3), lane = (int)((idx >> 2) & 31);
    const long long bk = idx >> 7;
    const int ks = (int)(bk % KS), b = (int)(bk / KS);
    const int g = lane >> 2, t = lane & 3;
    const int row = b * 16 + g + ((j & 1) ? 8 : 0);
    const int col = ks * 16 + 2 * t + ((j & 2) ? 8 : 0);
    uint32_t v = 0;
    if (row < E)
      v = (uint32_t)w[(size_t)row * H + col] | ((uint32_t)w[(size_t)row * H + col + 1] << 16);
    out[idx] = v;
  }
}

static int slice_geom(int group, int has_zeros, TileGeom* tg) {
  if (group != 32 && group != 64 && group != 128) return 1;
  if (tile_geom(kSliceK, group, has_zeros, tg)) return 1;
  const uint32_t end = tg->off_zero + (has_zeros ? (uint32_t)tg->Gr * 8u : 0u);
  tg->rec_bytes = (end + 15u) / 16u * 16u;
  return 0;
}

// ====================================================================== host side
static inline uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct StackScratch {
  size_t barrier, acc, qkv, h1, total;
};

static StackScratch stack_scratch(int T, int H, int qkv_R) {
  StackScratch s;
  size_t off = 0;
  s.barrier = off;
  off += 256;
  s.acc = off;  // right after the barrier counter: one memset zeroes both
  off += align_up((size_t)3 * T * H * 8, 256);
  s.qkv = off;
  off += align_up((size_t)T * (qkv_R > 0 ? qkv_R : 1) * 2, 256);
  s.h1 = off;
  off += align_up((size_t)T * H * 2, 256);
  s.total = off;
  return s;
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_down_slices_bytes(int32_t E, int32_t H, int32_t I, int32_t group,
                                        int has_zeros, size_t* bytes) {
  if (!bytes || E < 1 || H < 16 || (H & 15) || I < kSliceK || (I % kSliceK)) return DUPLEX_ERR_ARG;
  TileGeom tg;
  if (slice_geom(group, has_zeros, &tg)) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = (size_t)E * (I / kSliceK) * (H / 16) * tg.rec_bytes;
  return DUPLEX_OK;
}

extern "C" int duplex_repack_down_slices(const int32_t* packed, const void* scale,
                                         const int32_t* zeros, int scale_dtype, int32_t E,
                                         int32_t H, int32_t I, int32_t group, void* out,
                                         size_t out_bytes, void* stream) {
  size_t need = 0;
  int rc = duplex_down_slices_bytes(E, H, I, group, zeros != nullptr, &need);
  if (rc) return rc;
  if (!packed || !scale || !out) return DUPLEX_ERR_ARG;
  if (out_bytes < need) return DUPLEX_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(out) & 15u) return DUPLEX_ERR_ALIGN;
  TileGeom tg;
  slice_geom(group, zeros != nullptr, &tg);
  const int G = I / group, GZ = (G + 7) / 8;
  const long long words = (long long)(need / 4);
  long long blocks = (words + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  cudaStream_t st = (cudaStream_t)stream;
  if (scale_dtype == DUPLEX_DTYPE_F16)
    slice_repack_kernel<__half><<<(int)blocks, 256, 0, st>>>(
        packed, reinterpret_cast<const __half*>(scale), zeros, E, H, I, G, GZ, tg,
        reinterpret_cast<uint32_t*>(out));
  else if (scale_dtype == DUPLEX_DTYPE_BF16)
    slice_repack_kernel<__nv_bfloat16><<<(int)blocks, 256, 0, st>>>(
        packed, reinterpret_cast<const __nv_bfloat16*>(scale), zeros, E, H, I, G, GZ, tg,
        reinterpret_cast<uint32_t*>(out));
  else
    return DUPLEX_ERR_DTYPE;
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_gate_records_bytes(int32_t E, int32_t H, size_t* bytes) {
  if (!bytes || E < 1 || H < 16 || (H & 15)) return DUPLEX_ERR_ARG;
  *bytes = (size_t)((E + 15) / 16) * (H / 16) * 512;
  return DUPLEX_OK;
}

extern "C" int duplex_repack_gate_records(const void* gate_w, int dtype, int32_t E, int32_t H,
                                          void* out, size_t out_bytes, void* stream) {
  size_t need = 0;
  int rc = duplex_gate_records_bytes(E, H, &need);
  if (rc) return rc;
  if (!gate_w || !out) return DUPLEX_ERR_ARG;
  if (dtype != DUPLEX_DTYPE_F16 && dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (out_bytes < need) return DUPLEX_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(out) & 15u) return DUPLEX_ERR_ALIGN;
  const long long words = (long long)(need / 4);
  long long blocks = (words + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  gate_repack_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint16_t*>(gate_w), E, H, reinterpret_cast<uint32_t*>(out));
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_stack_workspace_bytes(int32_t T, int32_t H, int32_t E, int32_t I,
                                            int32_t top_k, int32_t qkv_R, size_t* bytes) {
  if (!bytes || T < 1 || H < 1 || E < 1 || I < 1 || top_k < 1) return DUPLEX_ERR_ARG;
  *bytes = stack_scratch(T, H, qkv_R).total;
  return DUPLEX_OK;
}

extern "C" int duplex_stack_forward(const duplex_stack_layer* layers, int32_t n_layers,
                                    int32_t has_attn, int32_t moe_residual, const void* x_in,
                                    void* out, int act_dtype, int scale_dtype, int has_zeros,
                                    int32_t T, int32_t H, int32_t E, int32_t I, int32_t top_k,
                                    int32_t norm_topk, int32_t qkv_R, int32_t q_dim,
                                    int32_t group, float rms_eps, void* workspace,
                                    size_t workspace_bytes, int64_t wait_limit_cycles,
                                    int32_t test_flags, int32_t* err, void* stream) {
  if (!layers || n_layers < 1 || n_layers > 255 || !x_in || !out || !workspace || !err)
    return DUPLEX_ERR_ARG;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  // H: whole 16-row down records per CTA, at most kMaxRecPerWarp per warp; I: whole slices
  if (H % (16 * kCS) || H > 16 * kCS * kCW * kMaxRecPerWarp || I % kSliceK || I < kSliceK)
    return DUPLEX_ERR_UNSUPPORTED;
  StackParams p = {};
  if (tile_geom(H, group, has_zeros, &p.tgu) || slice_geom(group, has_zeros, &p.tks))
    return DUPLEX_ERR_UNSUPPORTED;
  p.has_attn = has_attn ? 1 : 0;
  if (p.has_attn) {
    if (qkv_R < 16 || (qkv_R & 15) || q_dim < 64 || (q_dim & 63) || q_dim > qkv_R)
      return DUPLEX_ERR_UNSUPPORTED;
    if (tile_geom(H, group, has_zeros, &p.tq) || tile_geom(q_dim, group, has_zeros, &p.to))
      return DUPLEX_ERR_UNSUPPORTED;
  }
  const StackScratch L = stack_scratch(T, H, p.has_attn ? qkv_R : 0);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(x_in) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return DUPLEX_ERR_ALIGN;
  const int maxK = p.has_attn && q_dim > H ? q_dim : H;
  if (T * maxK > kMaxChunks * 8 * kConsumers) return DUPLEX_ERR_UNSUPPORTED;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  p.layers = layers;
  p.n_layers = n_layers;
  p.T = T; p.H = H; p.E = E; p.I = I; p.top_k = top_k; p.norm = norm_topk;
  p.q_dim = q_dim; p.qkv_R = qkv_R; p.moe_residual = moe_residual ? 1 : 0;
  p.RbQ = (qkv_R + 15) / 16; p.RbO = (H + 15) / 16;
  p.S = I / kSliceK;
  p.rrows = H / kCS;
  p.nblk = (E + 15) / 16;
  p.rms_eps = rms_eps;
  p.x_in = x_in; p.out = out;
  p.acc = reinterpret_cast<unsigned long long*>(ws + L.acc);
  p.qkv = ws + L.qkv;
  p.h1 = ws + L.h1;
  p.barrier = reinterpret_cast<unsigned*>(ws + L.barrier);
  p.err = err;
  p.wait_limit = wait_limit_cycles > 0 ? (long long)wait_limit_cycles : kWaitLimitCycles;
  p.test_flags = test_flags;
  // ring slot: the largest stage -- a q|k|v record, an o record, a gate|up record pair,
  // a CTA's down records of one slice; gate rows take as many rows as fit
  uint32_t slot = 2u * p.tgu.rec_bytes;
  if (p.has_attn) {
    slot = slot > p.tq.rec_bytes ? slot : p.tq.rec_bytes;
    slot = slot > p.to.rec_bytes ? slot : p.to.rec_bytes;
  }
  p.dn_bytes = (uint32_t)(p.rrows / 16) * p.tks.rec_bytes;
  slot = slot > 2u * p.dn_bytes ? slot : 2u * p.dn_bytes;
  slot = up(slot, 128);
  p.KS = H / 16;
  p.kps = (int)(slot / 512u);
  if (p.kps > p.KS) p.kps = p.KS;
  p.slot_bytes = slot;
  p.x_pitch = up((uint32_t)((maxK + 63) / 64 * 64) * 2u, 128) + 64u;
  const uint32_t gsum_bytes = (uint32_t)((maxK / 32) * 8 * 8);
  // items per batch: their deferred gate|up partials fit `red`, their rows fit xd
  int ib = kMaxBatch;
  const int by_red = (int)(kSRedBytes / 4) / (2 * kCW * T * 16);
  if (ib > by_red) ib = by_red;
  if (ib > kMaxBatchRows / T) ib = kMaxBatchRows / T;
  if (ib < 1) return DUPLEX_ERR_UNSUPPORTED;
  p.ib = ib;
  p.off_xd = up(kSFixedEnd, 128);
  p.off_av = p.off_xd + 2u * (uint32_t)(ib * T) * kXdPitch;           // column-sum partials
  p.off_dg = up(p.off_av + 2u * (uint32_t)ib * kCS * 8u * 8u, 16);
  p.off_gsum = up(p.off_dg + (uint32_t)ib * 4u * 8u * 8u, 128);
  p.off_h = up(p.off_gsum + gsum_bytes, 128);
  p.off_x = up(p.off_h + (uint32_t)T * (uint32_t)H * 2u, 128);
  p.off_ring = up(p.off_x + (uint32_t)T * p.x_pitch, 128);
  const size_t kMax = 227 * 1024;
  int ns = p.off_ring < kMax ? (int)((kMax - p.off_ring) / slot) : 0;
  if (ns > kSlotsMax) ns = kSlotsMax;
  if (ns < 2) return DUPLEX_ERR_UNSUPPORTED;
  p.nslots = ns;
  const size_t smem = p.off_ring + (size_t)ns * slot;

  cudaStream_t st = (cudaStream_t)stream;
  const bool g32 = group == 32;
  void (*kern)(StackParams);
  using H16 = __half;
  using B16 = __nv_bfloat16;
  if (act_dtype == DUPLEX_DTYPE_F16) {
    if (T == 1)
      kern = g32 ? stack_kernel<H16, H16, true, 1> : stack_kernel<H16, H16, false, 1>;
    else
      kern = g32 ? stack_kernel<H16, H16, true, 0> : stack_kernel<H16, H16, false, 0>;
  } else {
    if (T == 1)
      kern = g32 ? stack_kernel<B16, B16, true, 1> : stack_kernel<B16, B16, false, 1>;
    else
      kern = g32 ? stack_kernel<B16, B16, true, 0> : stack_kernel<B16, B16, false, 0>;
  }
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kMax);
  if (rc) return rc;
  // clusters of kCS CTAs, as many as can be resident at once: the grid barrier needs
  // every CTA running.  (No cooperative attribute: it adds only an up-front check,
  // and the profiler cannot launch cluster kernels with it.  A CTA that cannot start
  // in time -- another kernel holding SMs -- makes the barrier give up with
  // DUPLEX_DEVERR_TIMEOUT; it never hangs.)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(kCS * kMaxClusters);
  int nclusters = 0;
  rc = record_cuda(cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg));
  if (rc) return rc;
  if (nclusters < 1) return DUPLEX_ERR_UNSUPPORTED;
  if (nclusters > kMaxClusters) nclusters = kMaxClusters;
  cfg.gridDim = dim3(kCS * nclusters);
  // the barrier counter and the first layer's accumulator (the two later ones are
  // zeroed inside the launch)
  static_assert(sizeof(unsigned long long) == 8, "int64 accumulator");
  rc = record_cuda(cudaMemsetAsync(ws + L.barrier, 0, L.acc + (size_t)T * H * 8 - L.barrier, st));
  if (rc) return rc;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, p));
}
