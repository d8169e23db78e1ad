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
// separated by grid-wide barriers (a global arrival counter, bounded spin).  The
// producer warp walks the same schedule and streams the weight records of the
// CTA's tiles into a shared-memory ring with one bulk copy each, independent of
// the phase barriers: the static weights (q|k|v, o, gate rows) of the next
// phases are in flight while the current phase computes, and while the router
// decides it prefetches the next layer's static weights into L2.  Expert records
// follow as soon as this CTA has built the routing plan; the down projection's
// activation rows are copied once the gate|up phase has finished everywhere.
//
// Numerics are those of dq_gemv_kernel (gemv.cu) and route_kernel (moe.cu): offset
// dequantisation with a correction MMA for Q/O/G, exact (n - z) for N, fp32
// accumulation, logits rounded to the activation dtype, fp32 softmax, ties of the
// top-k to the lower expert id.
#include "gemv_core.cuh"
#include "moe.cuh"

#include <mutex>
#include <set>
#include <utility>

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);

struct StackParams {
  const duplex_stack_layer* layers;
  int n_layers, T, H, E, I, top_k, norm, q_dim, qkv_R, has_attn, moe_residual;
  TileGeom tq, to, tgu, tdn;
  int RbQ, RbO, RbGU, RbD;
  float rms_eps;
  const void* x_in;
  void* out;
  void* hbuf0;
  void* hbuf1;
  void* qkv;
  void* h1;
  void* act;
  float* logits;
  unsigned* barrier;
  int* err;
  int nslots, ups;
  uint32_t slot_bytes, off_ring, off_xsh, off_plain, off_xd, x_pitch, xd_pitch;
};

// fixed shared-memory map (bytes)
constexpr uint32_t kSFull = 0;        // 16 mbarriers
constexpr uint32_t kSEmpty = 128;     // 16 mbarriers
constexpr uint32_t kSPlan = 256;      // mbarrier: plan of the current layer ready
constexpr uint32_t kSActR = 264;      // mbarrier: gate|up finished grid-wide
constexpr uint32_t kSAbort = 272;     // int
constexpr uint32_t kSNUnits = 276;    // int
constexpr uint32_t kSCnt = 320;       // 8 ints (plan compaction)
constexpr uint32_t kSSel = 512;       // [8 tokens][8] ints
constexpr uint32_t kSW = 768;         // [8 tokens][8] floats
constexpr uint32_t kSUnitE = 1024;    // kMaxUnits ints
constexpr uint32_t kSUnitM = 1280;    // kMaxUnits uints
constexpr uint32_t kSUnitW = 1536;    // kMaxUnits * 8 floats
constexpr uint32_t kSLogit = 3584;    // [8][kMaxExperts] floats
constexpr uint32_t kSRed = kSLogit + 8 * kMaxExperts * 4;   // kCW * 8 * 32 floats
constexpr uint32_t kSCorr = kSRed + kCW * 8 * 32 * 4;       // correction table (dynamic size)
constexpr int kSlotsMax = 16;

DEVI bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

DEVI void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

DEVI unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer warps of every CTA.  Bounded: after ~2 s it
// records DUPLEX_DEVERR_TIMEOUT, sets the CTA's abort flag and stops waiting.
DEVI void grid_sync(const StackParams& p, unsigned& nb, int tid, volatile int* abort) {
  named_bar_sync(1, kConsumers);
  ++nb;
  if (tid == 0) {
    __threadfence();
    atomicAdd(p.barrier, 1u);
    const unsigned target = nb * gridDim.x;
    if (!*abort) {
      const long long t0 = clock64();
      while (ld_acquire_gpu(p.barrier) < target) {
        if (clock64() - t0 > kWaitLimitCycles) {
          *abort = 1;
          set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
          break;
        }
      }
    }
    __threadfence();
  }
  named_bar_sync(1, kConsumers);
}

template <typename T, typename S>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(const __grid_constant__ StackParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kSEmpty);
  uint64_t* plan_ready = reinterpret_cast<uint64_t*>(smem + kSPlan);
  uint64_t* act_ready = reinterpret_cast<uint64_t*>(smem + kSActR);
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
    mbar_init(act_ready, 1);
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
      if (j >= NS) {
        if (!mbar_wait_bounded(&empty[j % NS], (uint32_t)((j / NS) - 1) & 1u, abort_flag))
          if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
      }
    };
    auto slot_ptr = [&](int j) { return smem + p.off_ring + (uint32_t)(j % NS) * p.slot_bytes; };
    // one-copy stage (weights), the second arrival follows immediately
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
      if (!mbar_wait_bounded(plan_ready, (uint32_t)(l & 1), abort_flag))
        if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
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
                   ((size_t)unit_e[u] * p.RbGU + 2 * rbi) * p.tgu.rec_bytes,
               2u * p.tgu.rec_bytes);
      }
      // down: weights now, activation rows once gate|up has finished everywhere
      bool act_seen = false;
      int npend = 0;
      struct Pend { int seq, u0, cnt; } pq[kSlotsMax];
      auto flush = [&]() {
        fence_proxy_async_global();
        for (int q = 0; q < npend; ++q) {
          const Pend& pp = pq[q];
          uint8_t* dst = smem + p.off_ring + (uint32_t)(pp.seq % NS) * p.slot_bytes + p.off_xd;
          if (lane == 0)
            mbar_arrive_expect_tx(&full[pp.seq % NS], (uint32_t)(pp.cnt * p.T) * (uint32_t)p.I * 2u);
          __syncwarp();
          for (int r = lane; r < pp.cnt * p.T; r += 32) {
            const int us = r / p.T, n = r - us * p.T;
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.act) +
                                 ((size_t)(pp.u0 + us) * kMaxTokens + n) * p.I * 2;
            bulk_g2s(dst + (uint32_t)r * p.xd_pitch, src, (uint32_t)p.I * 2u, &full[pp.seq % NS]);
          }
          __syncwarp();
        }
        npend = 0;
      };
      const int nstg = (nu + p.ups - 1) / p.ups;
      for (int t = cta; t < p.RbD; t += G) {
        for (int s = 0; s < nstg; ++s) {
          if (!act_seen && npend > 0 && i >= NS &&
              !mbar_test(&empty[i % NS], (uint32_t)((i / NS) - 1) & 1u)) {
            if (!mbar_wait_bounded(act_ready, (uint32_t)(l & 1), abort_flag))
              if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
            act_seen = true;
            flush();
          }
          acquire(i);
          const int u0 = s * p.ups;
          const int cnt = (nu - u0) < p.ups ? (nu - u0) : p.ups;
          if (lane == 0) mbar_arrive_expect_tx(&full[i % NS], (uint32_t)cnt * p.tdn.rec_bytes);
          __syncwarp();
          if (lane < cnt)
            bulk_g2s_stream(slot_ptr(i) + (uint32_t)lane * p.tdn.rec_bytes,
                            reinterpret_cast<const uint8_t*>(L.dn_tiles) +
                                ((size_t)unit_e[u0 + lane] * p.RbD + t) * p.tdn.rec_bytes,
                            p.tdn.rec_bytes, &full[i % NS], pol);
          __syncwarp();
          pq[npend++] = Pend{i, u0, cnt};
          if (act_seen) flush();
          ++i;
        }
      }
      if (!act_seen) {
        if (!mbar_wait_bounded(act_ready, (uint32_t)(l & 1), abort_flag))
          if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
        flush();
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
          set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
          break;
        }
      }
    }
    return;
  }

  // ================================================================== consumers
  const int g = lane >> 2, t = lane & 3;
  float* red = reinterpret_cast<float*>(smem + kSRed);
  uint32_t* corr = reinterpret_cast<uint32_t*>(smem + kSCorr);
  uint8_t* xsh = smem + p.off_xsh;
  uint8_t* xplain = smem + p.off_plain;
  const bool xon = g < p.T;
  unsigned nb = 0;  // grid barriers passed
  int i = 0;        // stage sequence number

  auto wait_full = [&](int j) {
    if (!mbar_wait_bounded(&full[j % NS], (uint32_t)(j / NS) & 1u, abort_flag))
      if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
  };
  auto release = [&](int j) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[j % NS]);
  };
  auto slot_ptr = [&](int j) { return smem + p.off_ring + (uint32_t)(j % NS) * p.slot_bytes; };

  const uint8_t* h_prev = reinterpret_cast<const uint8_t*>(p.x_in);
  for (int l = 0; l < p.n_layers; ++l) {
    const duplex_stack_layer L = p.layers[l];
    uint8_t* h_out = reinterpret_cast<uint8_t*>(l == p.n_layers - 1 ? p.out
                                                : (l & 1) ? p.hbuf1 : p.hbuf0);
    const uint8_t* hm = h_prev;  // MoE input
    if (p.has_attn) {
      // ---------------------------------------------------------------- Q
      stage_x_shared<T, true>(xsh, p.x_pitch, h_prev, p.H, p.T, p.tq, p.rms_eps, red, tid, warp,
                              lane);
      build_corr<T>(corr, xsh, p.x_pitch, p.tq.npairs, p.T, tid);
      named_bar_sync(1, kConsumers);
      for (int tile = cta; tile < p.RbQ; tile += G, ++i) {
        wait_full(i);
        const int np = p.tq.npairs;
        const int lo = (warp * np) / kCW, hi = ((warp + 1) * np) / kCW;
        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
        consume_corr<T, S, false>(slot_ptr(i), p.tq, lo, hi, lane, xsh, p.x_pitch, corr, xon, a0, a1);
        release(i);
        float v, v2;
        reduce_tile(red, a0, a1, false, tid, warp, lane, v, v2);
        if (tid < 128) {
          const int n = tid >> 4, r = tid & 15, row = tile * 16 + r;
          if (n < p.T && row < p.qkv_R)
            reinterpret_cast<T*>(p.qkv)[(size_t)n * p.qkv_R + row] = from_f32<T>(v);
        }
        named_bar_sync(1, kConsumers);
      }
      grid_sync(p, nb, tid, abort_flag);
      // ---------------------------------------------------------------- O
      stage_x_shared<T, true>(xsh, p.x_pitch, reinterpret_cast<const uint8_t*>(p.qkv), p.qkv_R, p.T,
                              p.to, 0.f, red, tid, warp, lane);
      build_corr<T>(corr, xsh, p.x_pitch, p.to.npairs, p.T, tid);
      named_bar_sync(1, kConsumers);
      for (int tile = cta; tile < p.RbO; tile += G, ++i) {
        wait_full(i);
        const int np = p.to.npairs;
        const int lo = (warp * np) / kCW, hi = ((warp + 1) * np) / kCW;
        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
        consume_corr<T, S, false>(slot_ptr(i), p.to, lo, hi, lane, xsh, p.x_pitch, corr, xon, a0, a1);
        release(i);
        float v, v2;
        reduce_tile(red, a0, a1, false, tid, warp, lane, v, v2);
        if (tid < 128) {
          const int n = tid >> 4, r = tid & 15, row = tile * 16 + r;
          if (n < p.T && row < p.H) {
            const T res = __ldcg(reinterpret_cast<const T*>(h_prev) + (size_t)n * p.H + row);
            reinterpret_cast<T*>(p.h1)[(size_t)n * p.H + row] =
                from_f32<T>(to_f32<T>(from_f32<T>(v)) + to_f32<T>(res));
          }
        }
        named_bar_sync(1, kConsumers);
      }
      grid_sync(p, nb, tid, abort_flag);
      hm = reinterpret_cast<const uint8_t*>(p.h1);
    }
    // ------------------------------------------------------------------ R
    stage_x_shared<T, true>(xsh, p.x_pitch, hm, p.H, p.T, p.tgu, p.rms_eps, red, tid, warp, lane,
                            xplain);
    build_corr<T>(corr, xsh, p.x_pitch, p.tgu.npairs, p.T, tid);
    named_bar_sync(1, kConsumers);
    for (int e = cta; e < p.E; e += G, ++i) {
      wait_full(i);
      const uint4* wr = reinterpret_cast<const uint4*>(slot_ptr(i));
      const int nq = p.H >> 3;
      float part[kMaxTokens];
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) part[n] = 0.f;
      for (int q = tid; q < nq; q += kConsumers) {
        const uint4 wv = wr[q];
        const T* we = reinterpret_cast<const T*>(&wv);
#pragma unroll
        for (int n = 0; n < kMaxTokens; ++n) {
          if (n < p.T) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xplain + ((size_t)n * p.H + q * 8) * 2);
            const T* xe = reinterpret_cast<const T*>(&xv);
#pragma unroll
            for (int k = 0; k < 8; ++k) part[n] = fmaf(to_f32<T>(we[k]), to_f32<T>(xe[k]), part[n]);
          }
        }
      }
      release(i);
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) {
        float a = part[n];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) red[warp * 8 + n] = a;
      }
      named_bar_sync(1, kConsumers);
      if (tid < p.T) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) a += red[w * 8 + tid];
        if (L.gate_b) a += to_f32<T>(reinterpret_cast<const T*>(L.gate_b)[e]);
        p.logits[(size_t)tid * p.E + e] = to_f32<T>(from_f32<T>(a));
      }
      named_bar_sync(1, kConsumers);
    }
    grid_sync(p, nb, tid, abort_flag);
    // ------------------------------------------------------------------ D
    {
      float* ls = reinterpret_cast<float*>(smem + kSLogit);
      int* sel_s = reinterpret_cast<int*>(smem + kSSel);
      float* w_s = reinterpret_cast<float*>(smem + kSW);
      int* cnt = reinterpret_cast<int*>(smem + kSCnt);
      const int TE = p.T * p.E;
      for (int idx = tid; idx < TE; idx += kConsumers) ls[idx] = __ldcg(p.logits + idx);
      if (tid < kMaxTokens * 8) sel_s[tid] = 0;
      named_bar_sync(1, kConsumers);
      // rank of each logit within its token (ties -> lower expert id first)
      for (int idx = tid; idx < TE; idx += kConsumers) {
        const int tk = idx / p.E, e = idx - tk * p.E;
        const float v = ls[idx];
        const float* row = ls + tk * p.E;
        int rank = 0;
        for (int e2 = 0; e2 < p.E; ++e2) {
          const float v2 = row[e2];
          rank += (v2 > v) || (v2 == v && e2 < e);
        }
        if (rank < p.top_k) sel_s[tk * 8 + rank] = e;
      }
      named_bar_sync(1, kConsumers);
      if (warp < p.T) {
        const int tk = warp;
        const float* row = ls + tk * p.E;
        const float m = row[sel_s[tk * 8]];
        float den = 0.f;
        for (int e = lane; e < p.E; e += 32) den += expf(row[e] - m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
        if (lane == 0) {
          float pj[kMaxTopK], psum = 0.f;
          for (int j = 0; j < p.top_k; ++j) {
            pj[j] = expf(row[sel_s[tk * 8 + j]] - m) / den;
            psum += pj[j];
          }
          for (int j = 0; j < p.top_k; ++j) w_s[tk * 8 + j] = p.norm ? pj[j] / psum : pj[j];
        }
      }
      named_bar_sync(1, kConsumers);
      // unit plan: distinct selected experts in ascending id order
      const int nw = (p.E + 31) >> 5;
      uint32_t mask = 0;
      float wv[kMaxTokens];
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) wv[n] = 0.f;
      unsigned bal = 0;
      const int e = warp * 32 + lane;
      if (warp < nw) {
        if (e < p.E)
          for (int tk = 0; tk < p.T; ++tk)
            for (int j = 0; j < p.top_k; ++j)
              if (sel_s[tk * 8 + j] == e) {
                mask |= 1u << tk;
                wv[tk] = w_s[tk * 8 + j];
              }
        bal = __ballot_sync(0xffffffffu, mask != 0u);
        if (lane == 0) cnt[warp] = __popc(bal);
      }
      named_bar_sync(1, kConsumers);
      if (warp < nw && mask) {
        int base = 0;
        for (int w = 0; w < warp; ++w) base += cnt[w];
        const int pos = base + __popc(bal & ((1u << lane) - 1u));
        if (pos < kMaxUnits) {
          unit_e[pos] = e;
          unit_m[pos] = mask;
#pragma unroll
          for (int n = 0; n < kMaxTokens; ++n) unit_w[pos * kMaxTokens + n] = wv[n];
        }
      }
      if (tid == 0) {
        int tot = 0;
        for (int w = 0; w < nw; ++w) tot += cnt[w];
        *n_units_s = tot < kMaxUnits ? tot : kMaxUnits;
      }
      named_bar_sync(1, kConsumers);
      if (tid == 0) mbar_arrive(plan_ready);
    }
    const int nu = *n_units_s;
    // ------------------------------------------------------------------ G
    for (int tile = cta; tile < nu * perG; tile += G, ++i) {
      wait_full(i);
      const int np = p.tgu.npairs;
      const int lo = (warp * 2 * np) / kCW, hi = ((warp + 1) * 2 * np) / kCW;
      float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
      consume_corr<T, S, false>(slot_ptr(i), p.tgu, lo, hi, lane, xsh, p.x_pitch, corr, xon, a0, a1);
      release(i);
      float v, v2;
      reduce_tile(red, a0, a1, true, tid, warp, lane, v, v2);
      if (tid < 128) {
        const int n = tid >> 4, r = tid & 15;
        const int u = tile / perG, row = (tile - u * perG) * 16 + r;
        if (n < p.T) {
          const float a = ((unit_m[u] >> n) & 1u) ? silu_f32(v) * v2 : 0.f;
          reinterpret_cast<T*>(p.act)[((size_t)u * kMaxTokens + n) * p.I + frag_pos(row)] =
              from_f32<T>(a);
        }
      }
      named_bar_sync(1, kConsumers);
    }
    grid_sync(p, nb, tid, abort_flag);
    if (tid == 0) mbar_arrive(act_ready);
    // ------------------------------------------------------------------ N
    const int nstg = (nu + p.ups - 1) / p.ups;
    for (int tile = cta; tile < p.RbD; tile += G) {
      float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < nstg; ++s, ++i) {
        wait_full(i);
        const int u0 = s * p.ups;
        const int cnt = (nu - u0) < p.ups ? (nu - u0) : p.ups;
        const int np = p.tdn.npairs;
        const int items = cnt * np;
        const int lo = (warp * items) / kCW, hi = ((warp + 1) * items) / kCW;
        const uint8_t* st = slot_ptr(i);
        for (int it = lo; it < hi; ++it) {
          const int us = it / np, pp = it - us * np;
          const int u = u0 + us;
          const uint8_t* xrow = st + p.off_xd + (uint32_t)(us * p.T + g) * p.xd_pitch + (uint32_t)t * 16u;
          item_exact<T, S, false>(st + (uint32_t)us * p.tdn.rec_bytes, p.tdn, pp, lane, xrow, xon,
                                  false, unit_w[u * kMaxTokens + 2 * t],
                                  unit_w[u * kMaxTokens + 2 * t + 1], a0);
        }
        release(i);
      }
      float v, v2;
      reduce_tile(red, a0, a1, false, tid, warp, lane, v, v2);
      if (tid < 128) {
        const int n = tid >> 4, r = tid & 15, row = tile * 16 + r;
        if (n < p.T && row < p.H) {
          float y = v;
          if (p.moe_residual) y += to_f32<T>(__ldcg(reinterpret_cast<const T*>(hm) + (size_t)n * p.H + row));
          reinterpret_cast<T*>(h_out)[(size_t)n * p.H + row] = from_f32<T>(y);
        }
      }
      named_bar_sync(1, kConsumers);
    }
    grid_sync(p, nb, tid, abort_flag);
    h_prev = h_out;
  }
}

// ====================================================================== host side
static inline uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct StackScratch {
  size_t barrier, h0, h1buf, hm, qkv, act, logits, total;
};

static StackScratch stack_scratch(int T, int H, int E, int I, int top_k, int qkv_R) {
  StackScratch s;
  size_t off = 0;
  s.barrier = off; off += 256;
  s.h0 = off; off += align_up((size_t)T * H * 2, 256);
  s.h1buf = off; off += align_up((size_t)T * H * 2, 256);
  s.hm = off; off += align_up((size_t)T * H * 2, 256);
  s.qkv = off; off += align_up((size_t)T * (qkv_R > 0 ? qkv_R : 1) * 2, 256);
  int units = T * top_k < E ? T * top_k : E;
  if (units > kMaxUnits) units = kMaxUnits;
  s.act = off; off += align_up((size_t)units * kMaxTokens * I * 2, 256);
  s.logits = off; off += align_up((size_t)T * E * 4, 256);
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
  if (!layers || n_layers < 1 || !x_in || !out || !workspace) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  if ((H & 63) || (I & 63) || (group & 63)) return DUPLEX_ERR_UNSUPPORTED;
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
  const StackScratch L = stack_scratch(T, H, E, I, top_k, p.has_attn ? qkv_R : 0);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(x_in) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  p.layers = layers;
  p.n_layers = n_layers;
  p.T = T; p.H = H; p.E = E; p.I = I; p.top_k = top_k; p.norm = norm_topk;
  p.q_dim = q_dim; p.qkv_R = qkv_R; p.moe_residual = moe_residual ? 1 : 0;
  p.RbQ = (qkv_R + 15) / 16; p.RbO = (H + 15) / 16; p.RbGU = 2 * I / 16; p.RbD = (H + 15) / 16;
  p.rms_eps = rms_eps;
  p.x_in = x_in; p.out = out;
  p.hbuf0 = ws + L.h0; p.hbuf1 = ws + L.h1buf; p.h1 = ws + L.hm; p.qkv = ws + L.qkv;
  p.act = ws + L.act; p.logits = reinterpret_cast<float*>(ws + L.logits);
  p.barrier = reinterpret_cast<unsigned*>(ws + L.barrier);
  p.err = err;
  // shared memory: fixed map | correction table | staged x | plain x | ring
  int maxK = H, maxPairs = p.tgu.npairs;
  if (p.has_attn) {
    if (p.to.K > maxK) maxK = p.to.K;
    if (p.to.npairs > maxPairs) maxPairs = p.to.npairs;
  }
  p.x_pitch = up((uint32_t)((maxK + 63) / 64 * 64) * 2u, 128) + 64u;
  const uint32_t off_corr_end = kSCorr + (uint32_t)maxPairs * 128u;
  p.off_xsh = up(off_corr_end, 128);
  p.off_plain = up(p.off_xsh + (uint32_t)T * p.x_pitch, 128);
  p.off_ring = up(p.off_plain + (uint32_t)T * H * 2u, 128);
  // slot: the largest stage -- a q|k|v record, an o record, a gate row, a gate|up
  // record pair, or `ups` down records with their activation rows
  uint32_t slot = 2u * p.tgu.rec_bytes;
  if (p.has_attn) {
    slot = slot > p.tq.rec_bytes ? slot : p.tq.rec_bytes;
    slot = slot > p.to.rec_bytes ? slot : p.to.rec_bytes;
  }
  slot = slot > (uint32_t)H * 2u ? slot : (uint32_t)H * 2u;
  p.xd_pitch = up((uint32_t)I * 2u, 128) + 64u;
  const uint32_t per_unit = p.tdn.rec_bytes + (uint32_t)T * p.xd_pitch;
  int ups = (int)(slot / per_unit);
  if (ups < 1) {
    ups = 1;
    slot = per_unit;
  }
  if (ups > 32) ups = 32;
  p.ups = ups;
  p.off_xd = up((uint32_t)ups * p.tdn.rec_bytes, 128);
  slot = up(slot > p.off_xd + (uint32_t)ups * T * p.xd_pitch ? slot
                                                           : p.off_xd + (uint32_t)ups * T * p.xd_pitch,
            128);
  p.slot_bytes = slot;
  const size_t kMax = 227 * 1024;
  int ns = (int)((kMax - p.off_ring) / slot);
  if (ns > kSlotsMax) ns = kSlotsMax;
  if (ns < 2) return DUPLEX_ERR_UNSUPPORTED;
  p.nslots = ns;
  const size_t smem = p.off_ring + (size_t)ns * slot;

  cudaStream_t st = (cudaStream_t)stream;
  void (*kern)(StackParams) = act_dtype == DUPLEX_DTYPE_F16 ? stack_kernel<__half, __half>
                                                            : stack_kernel<__nv_bfloat16, __nv_bfloat16>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kMax);
  if (rc) return rc;
  int occ = 0;
  rc = record_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));
  if (rc) return rc;
  if (occ < 1) return DUPLEX_ERR_UNSUPPORTED;
  rc = record_cuda(cudaMemsetAsync(ws + L.barrier, 0, 256, st));
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, p));
}
