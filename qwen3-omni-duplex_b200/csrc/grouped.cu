// Batched-decode MoE (config 3: tens to hundreds of tokens through one MoE layer).
//
//   1. router logits on the tensor cores (16 experts x 16 tokens per CTA);
//   2. top-k per token (one warp per token, warp max-reductions over order keys),
//      fp32 softmax, renormalised weights;
//   3. a stable counting sort of the T*k (token, slot) assignments by expert and
//      the unit list: each expert's tokens split into units of <= kGTok;
//   4. the expert kernel: one CTA per unit streams its expert's gate|up and down
//      tile records exactly once (one bulk copy per stage, a 2-slot ring), keeps
//      the unit's tokens and the SiLU(gate)*up intermediate in shared memory, and
//      applies each dequantised weight fragment to up to three 8-token MMA column
//      blocks; it writes each (token, slot)'s expert output in fp32;
//   5. the combine: out[t] = sum over the slots, in selection order, of the routing
//      weight times the slot's expert output (+ residual), one rounding.
//
// Numerics match the decode path: offset dequantisation with the exact fp32 group
// correction, fp32 accumulation, logits rounded to the activation type, ties of
// the top-k to the lower expert id, the intermediate rounded to the activation
// type.  Every reduction runs in a fixed order.
#include "gemv_core.cuh"
#include "moe.cuh"
#include "topk.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);

constexpr int kGTok = 20;    // tokens of one expert unit
constexpr int kGNB = 3;      // 8-token MMA column blocks (kGNB * 8 >= kGTok)
constexpr int kGPad = 24;    // token slots per pair in the correction sums
constexpr int kGMaxT = 512;  // tokens per call
constexpr int kGSmemMax = 227 * 1024;

// ------------------------------------------------------------------ 1. router
// logits[t][e] = round_T(x[t] . gate_w[e] (+ b[e])): a CTA takes 16 experts x 16
// tokens, its 8 warps split K into k16 steps (ldmatrix + mma.sync, fp32).
template <typename T>
__global__ void __launch_bounds__(256) g_router_kernel(const T* x, const T* gw, const T* gb, int nT,
                                                       int E, int H, float* logits) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t pitch = (uint32_t)H * 2u + 16u;  // 16-byte skew: conflict-free ldmatrix
  uint8_t* ws = smem;
  uint8_t* xs = smem + 16 * pitch;
  float* red = reinterpret_cast<float*>(smem + 32 * pitch);  // [8 warps][16][16]
  const int e0 = blockIdx.x * 16, t0 = blockIdx.y * 16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nq = H >> 3;
  for (int idx = tid; idx < 32 * nq; idx += 256) {
    const int r = idx / nq, q = idx - r * nq;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < 16) {
      if (e0 + r < E) v = __ldg(reinterpret_cast<const uint4*>(gw + (size_t)(e0 + r) * H) + q);
    } else if (t0 + r - 16 < nT) {
      v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + r - 16) * H) + q);
    }
    *reinterpret_cast<uint4*>(smem + r * pitch + q * 16) = v;
  }
  __syncthreads();
  float acc[2][4];
  zero4(acc[0]);
  zero4(acc[1]);
  for (int k = warp; k < (H >> 4); k += 8) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(a0, a1, a2, a3, smem_u32(ws + (lane & 15) * pitch + k * 32 + (lane >> 4) * 16));
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      uint32_t b0, b1;
      ldsm_x2(b0, b1, smem_u32(xs + (nb * 8 + (lane & 7)) * pitch + k * 32 + ((lane >> 3) & 1) * 16));
      MmaOp<T>::run(acc[nb], a0, a1, a2, a3, b0, b1);
    }
  }
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nb = 0; nb < 2; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q)
      red[warp * 256 + (g + (q >> 1) * 8) * 16 + nb * 8 + 2 * t + (q & 1)] = acc[nb][q];
  __syncthreads();
  const int el = tid >> 4, tl = tid & 15;
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) s += red[w * 256 + tid];
  if (e0 + el < E && t0 + tl < nT) {
    if (gb) s += to_f32<T>(gb[e0 + el]);
    logits[(size_t)(t0 + tl) * E + e0 + el] = to_f32<T>(from_f32<T>(s));
  }
}

// ------------------------------------------------------------------ 2. top-k
// One warp per token (E <= 256: lane holds experts lane + 32 i): k rounds of a warp
// max-reduction over the order keys select the top k in descending order; softmax
// in fp32 over all experts; the top-k probabilities renormalised (their sum in
// selection order).
template <typename T>
__global__ void __launch_bounds__(512) g_topk_kernel(const float* logits, int nT, int E, int top_k,
                                                     int norm, int* sel, float* w, int32_t* sel_out,
                                                     float* w_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 16 + warp;
  if (t >= nT) return;  // whole warp
  const float* row = logits + (size_t)t * E;
  uint32_t key[8];
  float lv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    lv[i] = e < E ? row[e] : 0.f;
    key[i] = e < E ? order_key<T>(lv[i], e) : 0u;
  }
  int sj[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    sj[j] = 0;
    if (j < top_k) {
      uint32_t lm = 0u;
#pragma unroll
      for (int i = 0; i < 8; ++i) lm = key[i] > lm ? key[i] : lm;
      const uint32_t km = __reduce_max_sync(0xffffffffu, lm);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (key[i] == km) key[i] = 0u;
      const int e = key_expert(km);
      sj[j] = (km == 0u || e >= E) ? 0 : e;
    }
  }
  const float m = row[sj[0]];
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane + 32 * i < E) den += expf(lv[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  int ej = 0;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j)
    if (j == lane) ej = sj[j];
  const float pj = lane < top_k ? expf(row[ej] - m) / den : 0.f;
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    const float v = __shfl_sync(0xffffffffu, pj, j);
    if (j < top_k) psum += v;
  }
  if (lane < top_k) {
    const float wj = norm ? pj / psum : pj;
    sel[(size_t)t * top_k + lane] = ej;
    w[(size_t)t * top_k + lane] = wj;
    if (sel_out) sel_out[(size_t)t * top_k + lane] = ej;
    if (w_out) w_out[(size_t)t * top_k + lane] = wj;
  }
}

// ------------------------------------------------------------------ 3. bucketing
// Stable counting sort of the T*k assignments by expert (within an expert: token,
// then slot) into assign[] = token << 3 | slot, and the unit list: an expert's n
// assignments split into ceil(n / kGTok) units of near-equal size, units[u] =
// (expert, first assignment, count).  One CTA of 512 threads; chunks of 32
// assignments per warp (__match_any_sync gives ranks within a chunk).  Out-of-range
// expert ids are clamped to 0 and flagged.
__global__ void __launch_bounds__(512) g_bucket_kernel(const int* sel, int nT, int E, int top_k,
                                                       int* assign, int* units, int* n_units,
                                                       int max_units, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int N = nT * top_k, nch = (N + 31) >> 5;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t c_bytes = ((uint32_t)(nch * E) + 15u) & ~15u;
  const uint32_t p_bytes = ((uint32_t)(nch * E * 2) + 15u) & ~15u;
  uint8_t* cnt = smem;                                                  // [nch][E]
  uint16_t* pre = reinterpret_cast<uint16_t*>(smem + c_bytes);          // [nch][E]
  int* total = reinterpret_cast<int*>(smem + c_bytes + p_bytes);        // [E]
  int* base = total + kMaxExperts;                                         // [E]
  int* ubase = base + kMaxExperts;                                         // [E]
  for (int i = tid; i < nch * E; i += 512) cnt[i] = 0;
  __syncthreads();
  auto expert_of = [&](int a) {
    int e = a < N ? sel[a] : -1;
    if (a < N && (e < 0 || e >= E)) {
      set_error(err, DUPLEX_DEVERR_EXPERT);
      e = 0;
    }
    return e;
  };
  for (int c = warp; c < nch; c += 16) {
    const int a = c * 32 + lane;
    const int e = expert_of(a);
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(m) - 1) cnt[c * E + e] = (uint8_t)__popc(m);
  }
  __syncthreads();
  for (int e = tid; e < E; e += 512) {
    int s = 0;
    for (int c = 0; c < nch; ++c) {
      pre[c * E + e] = (uint16_t)s;
      s += cnt[c * E + e];
    }
    total[e] = s;
  }
  __syncthreads();
  if (tid == 0) {
    int b = 0, ub = 0;
    for (int e = 0; e < E; ++e) {
      base[e] = b;
      b += total[e];
      ubase[e] = ub;
      ub += (total[e] + kGTok - 1) / kGTok;
    }
    *n_units = ub < max_units ? ub : max_units;
  }
  __syncthreads();
  for (int c = warp; c < nch; c += 16) {
    const int a = c * 32 + lane;
    const int e = expert_of(a);
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int pos = base[e] + pre[c * E + e] + __popc(m & ((1u << lane) - 1u));
      assign[pos] = ((a / top_k) << 3) | (a % top_k);
    }
  }
  for (int e = tid; e < E; e += 512) {
    const int n = total[e];
    const int nu = (n + kGTok - 1) / kGTok;
    int off = 0;
    for (int k = 0; k < nu; ++k) {
      const int sz = n / nu + (k < n % nu ? 1 : 0);
      const int u = ubase[e] + k;
      if (u < max_units) {
        units[u * 3 + 0] = e;
        units[u * 3 + 1] = base[e] + off;
        units[u * 3 + 2] = sz;
      }
      off += sz;
    }
  }
}

// ------------------------------------------------------------------ 4. experts
struct GExpParams {
  int H, I, E, top_k;
  TileGeom tgu, tdn;
  const uint8_t* x;
  const uint8_t* gu_tiles;
  const uint8_t* dn_tiles;
  const int* assign;
  const int* units;
  const int* n_units;
  float* ypart;  // [T][k][H]
  int* err;
  uint32_t x_pitch, a_pitch, slot_bytes;
  uint32_t off_x, off_gx, off_a, off_ga, off_red, off_ring;
};

constexpr uint32_t kGFull = 0, kGEmpty = 16, kGAbort = 32, kGTokS = 64,
                   kGSlotS = 64 + 4 * kGTok, kGFixedEnd = 256;
static_assert(kGSlotS + 4 * kGTok <= kGFixedEnd, "fixed map");

// One warp's pairs [pb, pe) of one record against ntok staged token rows (up to
// kGNB blocks of 8): each pair's weights are dequantised once and applied to every
// block.  gsum: [pair][kGPad] float2 correction sums.
template <typename T, typename S>
DEVI void gmm_pairs(const uint8_t* rec, const TileGeom& tg, int pb, int pe, int lane,
                    const uint8_t* xsh, uint32_t pitch, const float2* gsum, int ntok,
                    float (&acc)[kGNB][4]) {
  const int g = lane >> 2, t = lane & 3;
  const int nbv = (ntok + 7) >> 3;
  const uint8_t* wp = rec + (((uint32_t)pb << 5) + lane) * 16u;
  int p = pb;
  while (p < pe) {
    const int grp = p >> tg.gshift;
    int pend = (grp + 1) << tg.gshift;
    if (pend > pe) pend = pe;
    float d[kGNB][4];
    float4 gs[kGNB];
#pragma unroll
    for (int nb = 0; nb < kGNB; ++nb) {
      zero4(d[nb]);
      gs[nb] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (; p < pend; ++p, wp += 512) {
      const uint4 w = *reinterpret_cast<const uint4*>(wp);
      uint32_t A0[4], B0[4], A1[4], B1[4];
      DqOff<T>::expand(w.x, w.y, A0, B0);
      DqOff<T>::expand(w.z, w.w, A1, B1);
#pragma unroll
      for (int nb = 0; nb < kGNB; ++nb) {
        if (nb < nbv) {  // warp-uniform
          const float4 gq = *reinterpret_cast<const float4*>(gsum + p * kGPad + nb * 8 + 2 * t);
          gs[nb].x += gq.x;
          gs[nb].y += gq.y;
          gs[nb].z += gq.z;
          gs[nb].w += gq.w;
          uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
          if (nb * 8 + g < ntok) {
            const uint8_t* xr = xsh + (uint32_t)(nb * 8 + g) * pitch + (uint32_t)t * 16u + (uint32_t)p * 128u;
            xa = *reinterpret_cast<const uint4*>(xr);
            xb = *reinterpret_cast<const uint4*>(xr + 64);
          }
          MmaOp<T>::run(d[nb], A0[0], A0[1], A0[2], A0[3], xa.x, xa.y);
          MmaOp<T>::run(d[nb], B0[0], B0[1], B0[2], B0[3], xa.z, xa.w);
          MmaOp<T>::run(d[nb], A1[0], A1[1], A1[2], A1[3], xb.x, xb.y);
          MmaOp<T>::run(d[nb], B1[0], B1[1], B1[2], B1[3], xb.z, xb.w);
        }
      }
    }
    const float zero4v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < kGNB; ++nb)
      if (nb < nbv) flush_group<S>(acc[nb], d[nb], zero4v, rec, tg, grp, g, gs[nb], 1.f, 1.f);
  }
}

// Partial sums of lane (g, t) -> red[warp][nb][q][lane]; read back per (row, token).
DEVI void put_acc(float* red, int warp, int lane, const float (&acc)[kGNB][4]) {
#pragma unroll
  for (int nb = 0; nb < kGNB; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) red[((warp * kGNB + nb) * 4 + q) * 32 + lane] = acc[nb][q];
}

DEVI int acc_at(int warp, int row, int tok) {
  const int g = row & 7, q = (row >> 3) * 2 + (tok & 1), t = (tok & 7) >> 1, nb = tok >> 3;
  return ((warp * kGNB + nb) * 4 + q) * 32 + g * 4 + t;
}

template <typename T, typename S>
__global__ void __launch_bounds__(kThreads, 1) g_expert_kernel(const __grid_constant__ GExpParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kGEmpty);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kGAbort);
  int* tok = reinterpret_cast<int*>(smem + kGTokS);
  int* slot = reinterpret_cast<int*>(smem + kGSlotS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int u = blockIdx.x;
  if (u >= *p.n_units) return;  // the whole CTA: units are fewer than the grid bound
  const int e = p.units[u * 3 + 0], first = p.units[u * 3 + 1];
  int n = p.units[u * 3 + 2];
  n = n < 0 ? 0 : (n > kGTok ? kGTok : n);
  const int perG = p.I >> 4;                // gate|up record pairs
  const int RbD = p.H >> 4;                 // down records
  const int nDN = (RbD + 3) >> 2;           // down stages of up to 4 records
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (tid < n) {
    const int a = p.assign[first + tid];
    tok[tid] = a >> 3;
    slot[tid] = a & 7;
  }
  __syncthreads();

  if (warp == kCW) {
    // ============================================================ producer
    // One thread.  After an abort nothing more is issued (a slot whose empty phase
    // did not complete is never re-armed); the copies already issued are drained.
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    int i = 0;
    auto issue = [&](const uint8_t* src, uint32_t bytes) {
      if (*abort_flag) return;
      if (i >= 2) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&empty[i & 1], (uint32_t)((i >> 1) - 1) & 1u)) {
          if (*abort_flag) return;
          if (clock64() - t0 > kWaitLimitCycles) {
            *abort_flag = 1;
            set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
            return;
          }
        }
      }
      mbar_arrive_expect_tx(&full[i & 1], bytes);
      bulk_g2s_stream(smem + p.off_ring + (uint32_t)(i & 1) * p.slot_bytes, src, bytes, &full[i & 1], pol);
      ++i;
    };
    for (int rb = 0; rb < perG; ++rb)
      issue(p.gu_tiles + ((size_t)e * 2 * perG + 2 * rb) * p.tgu.rec_bytes, 2u * p.tgu.rec_bytes);
    for (int s = 0; s < nDN; ++s) {
      const int cnt = RbD - 4 * s < 4 ? RbD - 4 * s : 4;
      issue(p.dn_tiles + ((size_t)e * RbD + 4 * s) * p.tdn.rec_bytes, (uint32_t)cnt * p.tdn.rec_bytes);
    }
    // drain: never leave while a copy may still target shared memory
    for (int j = i > 2 ? i - 2 : 0; j < i; ++j) {
      const long long t0 = clock64();
      while (!mbar_try_wait(&full[j & 1], (uint32_t)(j >> 1) & 1u))
        if (clock64() - t0 > 200000000LL) {
          set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
          break;
        }
    }
    return;
  }

  // ============================================================== consumers
  uint8_t* xsh = smem + p.off_x;
  float2* gx = reinterpret_cast<float2*>(smem + p.off_gx);
  uint8_t* act = smem + p.off_a;
  float2* ga = reinterpret_cast<float2*>(smem + p.off_ga);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  uint8_t* ring = smem + p.off_ring;
  const int H = p.H, I = p.I;
  int i = 0;
  auto wait_full = [&](int j) {
    if (*abort_flag) return;
    const long long t0 = clock64();
    while (!mbar_try_wait(&full[j & 1], (uint32_t)(j >> 1) & 1u)) {
      if (*abort_flag) return;
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort_flag = 1;
        set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
        return;
      }
    }
  };
  auto release = [&](int j) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[j & 1]);
  };

  // ---- the unit's token rows: fragment order (fp16: odd columns / 16), and the
  // per-pair correction sums (zero for absent tokens)
  {
    const int nq = H >> 3, total = n * nq;
    for (int base = 0; base < total + (kConsumers - 1) && base < total; base += kConsumers) {
      const int idx = base + tid;
      float se = 0.f, so = 0.f;
      int r = 0, q = 0;
      if (idx < total) {
        r = idx / nq;
        q = idx - r * nq;
        uint4 o = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)tok[r] * H * 2) + q);
        o = to_frag_order(o);
        if (DqOff<T>::kOddDiv16) {
          const __half2 q16 = __float2half2_rn(0.0625f);
          __half2 hy = __hmul2(*reinterpret_cast<__half2*>(&o.y), q16);
          __half2 hw = __hmul2(*reinterpret_cast<__half2*>(&o.w), q16);
          o.y = *reinterpret_cast<uint32_t*>(&hy);
          o.w = *reinterpret_cast<uint32_t*>(&hw);
        }
        *reinterpret_cast<uint4*>(xsh + (uint32_t)r * p.x_pitch + (uint32_t)q * 16u) = o;
        const T* v = reinterpret_cast<const T*>(&o);
        se = (to_f32<T>(v[0]) + to_f32<T>(v[1])) + (to_f32<T>(v[4]) + to_f32<T>(v[5]));
        so = (to_f32<T>(v[2]) + to_f32<T>(v[3])) + (to_f32<T>(v[6]) + to_f32<T>(v[7]));
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        so += __shfl_xor_sync(0xffffffffu, so, o);
      }
      if (idx < total && (q & 7) == 0) {
        const float P = DqOff<T>::kOddDiv16 ? 1024.f * (se + so) : 128.f * (se + so);
        const float Q = DqOff<T>::kOddDiv16 ? fmaf(16.f, so, se) : se + so;
        gx[(q >> 3) * kGPad + r] = make_float2(P, Q);
      }
    }
    const int np = p.tgu.npairs;
    for (int idx = tid; idx < np * kGPad; idx += kConsumers)
      if (idx % kGPad >= n) gx[idx] = make_float2(0.f, 0.f);
  }
  named_bar_sync(1, kConsumers);

  // ---- gate|up: warps 0-7 the gate record, 8-15 the up record, 8-way K split
  {
    const int rec = warp >> 3, kw = warp & 7, np = p.tgu.npairs;
    for (int rb = 0; rb < perG; ++rb, ++i) {
      wait_full(i);
      const uint8_t* st = ring + (uint32_t)(i & 1) * p.slot_bytes + (uint32_t)rec * p.tgu.rec_bytes;
      float acc[kGNB][4];
#pragma unroll
      for (int nb = 0; nb < kGNB; ++nb) zero4(acc[nb]);
      gmm_pairs<T, S>(st, p.tgu, (kw * np) >> 3, ((kw + 1) * np) >> 3, lane, xsh, p.x_pitch, gx, n,
                      acc);
      release(i);
      put_acc(red, warp, lane, acc);
      named_bar_sync(1, kConsumers);
      for (int o = tid; o < 16 * n; o += kConsumers) {
        const int row = o & 15, tk = o >> 4;
        float gsum_ = 0.f, usum = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          gsum_ += red[acc_at(w, row, tk)];
          usum += red[acc_at(8 + w, row, tk)];
        }
        const int col = rb * 16 + row;
        T a = from_f32<T>(silu_f32(gsum_) * usum);
        if (DqOff<T>::kOddDiv16 && (col & 1)) a = from_f32<T>(to_f32<T>(a) * 0.0625f);
        reinterpret_cast<T*>(act + (uint32_t)tk * p.a_pitch)[frag_pos(col)] = a;
      }
      named_bar_sync(1, kConsumers);
    }
  }

  // ---- correction sums of the intermediate
  {
    const int np = p.tdn.npairs;
    for (int idx = tid; idx < np * kGPad; idx += kConsumers) {
      const int pp = idx / kGPad, tk = idx - pp * kGPad;
      float se = 0.f, so = 0.f;
      if (tk < n) {
        const uint8_t* rowp = act + (uint32_t)tk * p.a_pitch + (uint32_t)pp * 128u;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 o = *reinterpret_cast<const uint4*>(rowp + c * 16);
          const T* v = reinterpret_cast<const T*>(&o);
          se += (to_f32<T>(v[0]) + to_f32<T>(v[1])) + (to_f32<T>(v[4]) + to_f32<T>(v[5]));
          so += (to_f32<T>(v[2]) + to_f32<T>(v[3])) + (to_f32<T>(v[6]) + to_f32<T>(v[7]));
        }
      }
      const float P = DqOff<T>::kOddDiv16 ? 1024.f * (se + so) : 128.f * (se + so);
      const float Q = DqOff<T>::kOddDiv16 ? fmaf(16.f, so, se) : se + so;
      ga[idx] = make_float2(P, Q);
    }
  }
  named_bar_sync(1, kConsumers);

  // ---- down: 4 records per stage, 4 warps per record (K split)
  {
    const int q4 = warp >> 2, kp = warp & 3, np = p.tdn.npairs;
    for (int s = 0; s < nDN; ++s, ++i) {
      wait_full(i);
      const int cnt = RbD - 4 * s < 4 ? RbD - 4 * s : 4;
      float acc[kGNB][4];
#pragma unroll
      for (int nb = 0; nb < kGNB; ++nb) zero4(acc[nb]);
      if (q4 < cnt)
        gmm_pairs<T, S>(ring + (uint32_t)(i & 1) * p.slot_bytes + (uint32_t)q4 * p.tdn.rec_bytes, p.tdn,
                        (kp * np) >> 2, ((kp + 1) * np) >> 2, lane, act, p.a_pitch, ga, n, acc);
      release(i);
      put_acc(red, warp, lane, acc);
      named_bar_sync(1, kConsumers);
      for (int o = tid; o < cnt * 16 * n; o += kConsumers) {
        const int rq = o / n, tk = o - rq * n;  // rq = record * 16 + row
        const int rc = rq >> 4, row = rq & 15;
        float y = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) y += red[acc_at(rc * 4 + w, row, tk)];
        p.ypart[((size_t)tok[tk] * p.top_k + slot[tk]) * H + (4 * s + rc) * 16 + row] = y;
      }
      named_bar_sync(1, kConsumers);
    }
  }
  (void)I;
}

// ------------------------------------------------------------------ 5. combine
template <typename T>
__global__ void __launch_bounds__(256) g_combine_kernel(const float* ypart, const float* w, const T* residual,
                                                        int nT, int H, int top_k, T* out) {
  const size_t idx = (size_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (size_t)nT * H) return;
  const int t = (int)(idx / H), r = (int)(idx - (size_t)t * H);
  float s = 0.f;
  for (int j = 0; j < top_k; ++j) s = fmaf(w[(size_t)t * top_k + j], ypart[((size_t)t * top_k + j) * H + r], s);
  if (residual) s += to_f32<T>(residual[idx]);
  out[idx] = from_f32<T>(s);
}

// ====================================================================== host side
struct GScratch {
  size_t logits, sel, w, assign, units, n_units, ypart, total;
  int max_units;
};

static GScratch g_scratch(int T, int E, int H, int top_k) {
  GScratch s;
  size_t off = 0;
  s.max_units = E + (T * top_k + kGTok - 1) / kGTok + 1;
  s.logits = off; off += align_up((size_t)T * E * 4, 256);
  s.sel = off; off += align_up((size_t)T * top_k * 4, 256);
  s.w = off; off += align_up((size_t)T * top_k * 4, 256);
  s.assign = off; off += align_up((size_t)T * top_k * 4, 256);
  s.units = off; off += align_up((size_t)s.max_units * 12, 256);
  s.n_units = off; off += 256;
  s.ypart = off; off += align_up((size_t)T * top_k * H * 4, 256);
  s.total = off;
  return s;
}

// Shared-memory map of the expert kernel for one geometry; false when it does not fit.
static bool g_layout(int H, int I, int group, int has_zeros, GExpParams* p, size_t* smem) {
  if ((H & 63) || (I & 63) || group < 64 || (group & (group - 1))) return false;
  if (32 * (H * 2 + 16) + 8 * 256 * 4 > kGSmemMax) return false;  // router tile
  if (tile_geom(H, group, has_zeros, &p->tgu) || tile_geom(I, group, has_zeros, &p->tdn)) return false;
  auto up = [](uint32_t v, uint32_t a) { return (v + a - 1) / a * a; };
  p->x_pitch = up((uint32_t)H * 2u, 128) + 64u;
  p->a_pitch = up((uint32_t)I * 2u, 128) + 64u;
  uint32_t slot = 2u * p->tgu.rec_bytes;
  if (slot < 4u * p->tdn.rec_bytes) slot = 4u * p->tdn.rec_bytes;
  p->slot_bytes = up(slot, 128);
  p->off_x = kGFixedEnd;
  p->off_gx = up(p->off_x + kGTok * p->x_pitch, 128);
  p->off_a = up(p->off_gx + (uint32_t)p->tgu.npairs * kGPad * 8u, 128);
  p->off_ga = up(p->off_a + kGTok * p->a_pitch, 128);
  p->off_red = up(p->off_ga + (uint32_t)p->tdn.npairs * kGPad * 8u, 128);
  p->off_ring = up(p->off_red + kCW * kGNB * 4 * 32 * 4, 128);
  *smem = p->off_ring + 2 * (size_t)p->slot_bytes;
  return *smem <= (size_t)kGSmemMax;
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_moe_grouped_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                                  int32_t top_k, int32_t group, int has_zeros,
                                                  size_t* bytes) {
  if (!bytes || T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 ||
      top_k > kMaxTopK || top_k > E || H < 1 || I < 1)
    return DUPLEX_ERR_ARG;
  GExpParams p = {};
  size_t smem = 0;
  if (!g_layout(H, I, group, has_zeros, &p, &smem)) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = g_scratch(T, E, H, top_k).total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_grouped(const void* x, int act_dtype, int32_t T, const void* gate_w,
                                  const void* gate_b, const float* logits_in, int32_t E, int32_t H,
                                  int32_t I, int32_t top_k, int32_t norm_topk, const void* gu_tiles,
                                  const void* dn_tiles, int scale_dtype, int has_zeros,
                                  int32_t group, const void* residual, void* out, float* w_out,
                                  int32_t* sel_out, void* workspace, size_t workspace_bytes,
                                  int32_t* err, void* stream) {
  if (!x || !out || !gu_tiles || !dn_tiles || !workspace || (!gate_w && !logits_in)) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  GExpParams p = {};
  size_t smem = 0;
  if (!g_layout(H, I, group, has_zeros, &p, &smem)) return DUPLEX_ERR_UNSUPPORTED;
  const GScratch L = g_scratch(T, E, H, top_k);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(gu_tiles) |
       reinterpret_cast<uintptr_t>(dn_tiles) | reinterpret_cast<uintptr_t>(gate_w) |
       reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(logits_in)) & 15u)
    return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* logits = logits_in ? const_cast<float*>(logits_in) : reinterpret_cast<float*>(ws + L.logits);
  int* sel = reinterpret_cast<int*>(ws + L.sel);
  float* w = reinterpret_cast<float*>(ws + L.w);
  cudaStream_t st = (cudaStream_t)stream;
  const bool f16 = act_dtype == DUPLEX_DTYPE_F16;
  int rc;
  // 1. router
  if (!logits_in) {
    const int smem = 32 * (H * 2 + 16) + 8 * 256 * 4;
    void (*rk)(const __half*, const __half*, const __half*, int, int, int, float*) = g_router_kernel<__half>;
    void (*rkb)(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, int, int, int, float*) =
        g_router_kernel<__nv_bfloat16>;
    const void* fn = f16 ? reinterpret_cast<const void*>(rk) : reinterpret_cast<const void*>(rkb);
    // the attribute is set once per kernel (to the ceiling), whatever this call's size
    if (smem > kGSmemMax) return DUPLEX_ERR_UNSUPPORTED;
    if ((rc = ensure_smem_attr(fn, kGSmemMax))) return rc;
    const dim3 grid((E + 15) / 16, (T + 15) / 16);
    if (f16)
      rk<<<grid, 256, smem, st>>>(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(gate_w),
                                  reinterpret_cast<const __half*>(gate_b), T, E, H, logits);
    else
      rkb<<<grid, 256, smem, st>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                   reinterpret_cast<const __nv_bfloat16*>(gate_w),
                                   reinterpret_cast<const __nv_bfloat16*>(gate_b), T, E, H, logits);
    if ((rc = record_cuda(cudaGetLastError()))) return rc;
  }
  // 2. top-k
  if (f16)
    g_topk_kernel<__half><<<(T + 15) / 16, 512, 0, st>>>(logits, T, E, top_k, norm_topk, sel, w, sel_out, w_out);
  else
    g_topk_kernel<__nv_bfloat16><<<(T + 15) / 16, 512, 0, st>>>(logits, T, E, top_k, norm_topk, sel, w, sel_out,
                                                                w_out);
  if ((rc = record_cuda(cudaGetLastError()))) return rc;
  // 3. bucketing
  {
    const int N = T * top_k, nch = (N + 31) / 32;
    const int smem = (int)(align_up((size_t)nch * E, 16) + align_up((size_t)nch * E * 2, 16) +
                           3 * kMaxExperts * 4);
    if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(g_bucket_kernel), kGSmemMax))) return rc;
    g_bucket_kernel<<<1, 512, smem, st>>>(sel, T, E, top_k, reinterpret_cast<int*>(ws + L.assign),
                                          reinterpret_cast<int*>(ws + L.units),
                                          reinterpret_cast<int*>(ws + L.n_units), L.max_units, err);
    if ((rc = record_cuda(cudaGetLastError()))) return rc;
  }
  // 4. experts
  p.H = H; p.I = I; p.E = E; p.top_k = top_k;
  p.x = reinterpret_cast<const uint8_t*>(x);
  p.gu_tiles = reinterpret_cast<const uint8_t*>(gu_tiles);
  p.dn_tiles = reinterpret_cast<const uint8_t*>(dn_tiles);
  p.assign = reinterpret_cast<const int*>(ws + L.assign);
  p.units = reinterpret_cast<const int*>(ws + L.units);
  p.n_units = reinterpret_cast<const int*>(ws + L.n_units);
  p.ypart = reinterpret_cast<float*>(ws + L.ypart);
  p.err = err;
  void (*ek)(GExpParams) = f16 ? g_expert_kernel<__half, __half> : g_expert_kernel<__nv_bfloat16, __nv_bfloat16>;
  if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(ek), kGSmemMax))) return rc;
  ek<<<L.max_units, kThreads, smem, st>>>(p);
  if ((rc = record_cuda(cudaGetLastError()))) return rc;
  // 5. combine
  const size_t n_out = (size_t)T * H;
  const unsigned blocks = (unsigned)((n_out + 255) / 256);
  if (f16)
    g_combine_kernel<__half><<<blocks, 256, 0, st>>>(reinterpret_cast<const float*>(ws + L.ypart), w,
                                                      reinterpret_cast<const __half*>(residual), T, H, top_k,
                                                      reinterpret_cast<__half*>(out));
  else
    g_combine_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(reinterpret_cast<const float*>(ws + L.ypart), w,
                                                             reinterpret_cast<const __nv_bfloat16*>(residual),
                                                             T, H, top_k, reinterpret_cast<__nv_bfloat16*>(out));
  return record_cuda(cudaGetLastError());
}
