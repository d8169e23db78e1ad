// Batched-decode MoE (config 3: tens to hundreds of tokens through one MoE layer).
//
//   1. router logits on the tensor cores (16 experts x 16 tokens per CTA);
//   2. top-k per token (one warp per token, warp max-reductions over order keys),
//      fp32 softmax, renormalised weights;
//   3. a stable counting sort of the T*k (token, slot) assignments by expert and
//      the unit list: each expert's tokens split into units of <= tcap (8, 16 or 20,
//      from the expected tokens per expert);
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
#include "umma.cuh"

#include <initializer_list>
#include <type_traits>

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);

constexpr int kGTok = 20;    // tokens of one expert unit at most (the per-call cap tcap <= kGTok)
constexpr int kGNB = 3;      // 8-token MMA column blocks at most
static_assert(kGNB * 8 >= kGTok, "a unit's tokens fit the MMA column blocks");
constexpr int kGPad = 24;    // token slots per pair in the correction sums
constexpr int kGMaxT = 512;  // tokens per call
constexpr int kGSmemMax = 227 * 1024;  // dynamic shared memory of every kernel here (no static)
// router CTA: 32 operand rows, the partials of 8 warps, its barrier
constexpr int g_router_smem(int H) { return 32 * (H * 2 + 16) + 8 * 256 * 4 + 16; }

// ------------------------------------------------------------------ 1. router
// logits[t][e] = round_T(x[t] . gate_w[e] (+ b[e])): a CTA takes 16 experts x 16
// tokens; its 32 operand rows arrive by bulk copies (one thread issues them, rows past
// E or T are zero-filled), then 8 warps split K into k16 steps (ldmatrix + mma.sync,
// fp32) and the partials are added in warp order.
template <typename T>
__global__ void __launch_bounds__(256) g_router_kernel(const T* x, const T* gw, const T* gb, int nT,
                                                       int E, int H, float* logits, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t pitch = (uint32_t)H * 2u + 16u;  // 16-byte skew: conflict-free ldmatrix
  uint8_t* ws = smem;
  uint8_t* xs = smem + 16 * pitch;
  float* red = reinterpret_cast<float*>(smem + 32 * pitch);  // [8 warps][16][16]
  uint64_t& bar = *reinterpret_cast<uint64_t*>(smem + 32 * pitch + 8 * 256 * 4);
  const int e0 = blockIdx.x * 16, t0 = blockIdx.y * 16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ne = E - e0 < 16 ? E - e0 : 16, nt = nT - t0 < 16 ? nT - t0 : 16;
  const uint32_t row_bytes = (uint32_t)H * 2u;
  pdl_launch_dependents();
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, (uint32_t)(ne + nt) * row_bytes);
    for (int r = 0; r < ne; ++r) bulk_g2s(ws + r * pitch, gw + (size_t)(e0 + r) * H, row_bytes, &bar);
    for (int r = 0; r < nt; ++r) bulk_g2s(xs + r * pitch, x + (size_t)(t0 + r) * H, row_bytes, &bar);
  }
  const int nq = H >> 3;
  for (int idx = tid; idx < 32 * nq; idx += 256) {
    const int r = idx / nq, q = idx - r * nq;
    if ((r < 16 && r >= ne) || (r >= 16 && r - 16 >= nt))
      *reinterpret_cast<uint4*>(smem + r * pitch + q * 16) = make_uint4(0, 0, 0, 0);
  }
  {
    const long long start = clock64();
    while (!mbar_try_wait(&bar, 0)) {
      if (clock64() - start > kWaitLimitCycles) {
        set_error(err, DUPLEX_DEVERR_TIMEOUT);
        break;
      }
    }
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
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[w * 256 + tid];
  if (el < ne && tl < nt) {
    if (gb) sum += to_f32<T>(gb[e0 + el]);
    logits[(size_t)(t0 + tl) * E + e0 + el] = to_f32<T>(from_f32<T>(sum));
  }
}

// ------------------------------------------------------------------ 2. top-k
// One warp per token (E <= 256: lane holds experts lane + 32 i): k rounds of a warp
// max-reduction over the order keys select the top k in descending order; softmax
// in fp32 over all experts; the top-k probabilities renormalised (their sum in
// selection order).
// PACK: the warp also writes its token's exchange row in pack: the token (2 H bytes,
// copied from x), its k expert ids (int32), its k weights (fp32), row_bytes apart.
template <typename T, bool PACK>
__global__ void __launch_bounds__(512) g_topk_kernel(const float* logits, int nT, int E, int top_k,
                                                     int norm, int* sel, float* w, int32_t* sel_out,
                                                     float* w_out, const T* x, int H, uint8_t* pack,
                                                     int64_t row_bytes) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 16 + warp;
  pdl_launch_dependents();
  pdl_wait();
  if (t >= nT) return;  // whole warp
  if constexpr (PACK) {  // the token's bytes first, while the logits loads are in flight
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(pack + (size_t)t * row_bytes);
    for (int q = lane; q < (H >> 3); q += 32) dst[q] = __ldg(src + q);
  }
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
  int ej = 0;  // lane j's pick
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
      ej = lane == j ? sj[j] : ej;  // taken here: read after the loop, the last pick came out 0
    }
  }
  const float m = row[sj[0]];
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane + 32 * i < E) den += expf(lv[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  const float pj = lane < top_k ? expf(row[ej] - m) / den : 0.f;
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    const float v = __shfl_sync(0xffffffffu, pj, j);
    if (j < top_k) psum += v;
  }
  if (lane < top_k) {
    const float wj = norm ? pj / psum : pj;
    if (sel) sel[(size_t)t * top_k + lane] = ej;
    if (w) w[(size_t)t * top_k + lane] = wj;
    if (sel_out) sel_out[(size_t)t * top_k + lane] = ej;
    if (w_out) w_out[(size_t)t * top_k + lane] = wj;
    if constexpr (PACK) {
      uint8_t* meta = pack + (size_t)t * row_bytes + (size_t)H * 2;
      reinterpret_cast<int32_t*>(meta)[lane] = ej;
      reinterpret_cast<float*>(meta + 4 * top_k)[lane] = wj;
    }
  }
}

// ------------------------------------------------------------------ 3. bucketing
// Stable counting sort of the T*k assignments by expert (within an expert: token,
// then slot) into assign[] = token << 3 | slot, and the unit list: an expert's n
// assignments split into ceil(n / tcap) units of near-equal size, units[u] =
// (expert, first assignment, count).  One CTA of 512 threads; chunks of 32
// assignments per warp (__match_any_sync gives ranks within a chunk).  Only experts
// [e_begin, e_begin + E) are bucketed (an expert-parallel rank's own); ids outside
// [0, E_total) are flagged in err and skipped.  Token t's ids are sel[t * sel_stride ..].
__global__ void __launch_bounds__(512) g_bucket_kernel(const int* sel, int sel_stride, int nT, int E, int top_k,
                                                       int tcap, int e_begin, int E_total, int* assign, int* units,
                                                       int* n_units, int max_units, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int N = nT * top_k, nch = (N + 31) >> 5;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t c_bytes = ((uint32_t)(nch * E) + 15u) & ~15u;
  const uint32_t p_bytes = ((uint32_t)(nch * E * 2) + 15u) & ~15u;
  pdl_launch_dependents();
  pdl_wait();
  uint8_t* cnt = smem;                                                  // [nch][E]
  uint16_t* pre = reinterpret_cast<uint16_t*>(smem + c_bytes);          // [nch][E]
  int* total = reinterpret_cast<int*>(smem + c_bytes + p_bytes);        // [E]
  int* base = total + kMaxExperts;                                         // [E]
  int* ubase = base + kMaxExperts;                                         // [E]
  int* sel_s = ubase + kMaxExperts + 16;                                   // [N]: after wsum
  for (int i = tid; i < nch * E; i += 512) cnt[i] = 0;
  // every selection into shared memory in one round of loads (both passes below read it)
  for (int a = tid; a < N; a += 512) {
    const int ta = a / top_k;
    sel_s[a] = sel[(size_t)ta * sel_stride + (a - ta * top_k)];
  }
  __syncthreads();
  // local expert of assignment a: ids outside [0, E_total) are flagged and skipped,
  // ids of other ranks' experts (outside [e_begin, e_begin + E)) are skipped
  auto expert_of = [&](int a) {
    if (a >= N) return -1;
    const int g = sel_s[a];
    if (g < 0 || g >= E_total) {
      set_error(err, DUPLEX_DEVERR_EXPERT);
      return -1;
    }
    const int e = g - e_begin;
    return (e < 0 || e >= E) ? -1 : e;
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
  {
    // exclusive scans of the assignment and unit counts over the experts (E <= 256:
    // warps 0-7, warp-level inclusive scans, then the warp totals in order)
    int* wsum = ubase + kMaxExperts;  // [2][8]
    int tot = 0, nun = 0, inc = 0, incu = 0;
    if (tid < 256) {
      tot = tid < E ? total[tid] : 0;
      nun = (tot + tcap - 1) / tcap;
      inc = tot;
      incu = nun;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc, o), b = __shfl_up_sync(0xffffffffu, incu, o);
        if (lane >= o) {
          inc += a;
          incu += b;
        }
      }
      if (lane == 31) {
        wsum[warp] = inc;
        wsum[8 + warp] = incu;
      }
    }
    __syncthreads();
    if (tid < 256) {
      for (int w = 0; w < warp; ++w) {
        inc += wsum[w];
        incu += wsum[8 + w];
      }
      if (tid < E) {
        base[tid] = inc - tot;
        ubase[tid] = incu - nun;
      }
      if (tid == 255) *n_units = incu < max_units ? incu : max_units;
    }
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
    const int nu = (n + tcap - 1) / tcap;
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
// Two persistent kernels, one CTA per SM, over flattened work lists so that every
// SM streams whatever the routing: gate|up items (unit, record pair) and down items
// (unit, stage of 8 down records).  A CTA takes a contiguous range of the list, so
// it re-stages a unit's token rows only when its range crosses into the next unit.
// One producer thread keeps a ring of bulk copies in flight; 16 consumer warps
// apply each dequantised weight fragment to the unit's NB = ceil(n / 8) 8-token MMA
// column blocks (NB dispatched per unit, warp-uniform).
//
// MMA columns of absent tokens (rows n .. 8 NB - 1 of the staged block) are never
// read back: each output column depends on its own token only, so those rows are
// neither zeroed nor masked (they lie inside this CTA's shared memory).
constexpr int kGMaxSlots = 8;
constexpr int kGDnRec = 8;  // down records per stage (one per warp of an 8-warp group)

struct GExpParams {
  int H, I, E, top_k, max_units;
  int tcap;        // tokens of one unit at most (<= kGTok)
  int red_floats;  // one warp group's partials: 8 warps x ceil(tcap / 8) blocks x 128
  TileGeom tgu, tdn;
  const uint8_t* x;
  size_t x_row_bytes;  // token rows of x this many bytes apart (2 H when packed)
  const uint8_t* gu_tiles;
  const uint8_t* dn_tiles;
  const int* assign;
  const int* units;
  const int* n_units;
  uint8_t* act;   // [T*k][I] SiLU(gate)*up per sorted assignment, fragment order
  float* ypart;   // [T][k][H]
  int* err;
  uint32_t x_pitch, a_pitch;
  // gate|up kernel map: token rows, per-pair and per-group correction sums, partials, ring
  uint32_t off_x, off_gx, off_gxg, off_red_a, off_ring_a, slot_a, smem_a;
  int ns_a;
  // down kernel map
  uint32_t off_a, off_ga, off_gag, off_ring_d, slot_d, smem_d;
  int ns_d;
};

constexpr uint32_t kGFull = 0, kGEmpty = 8 * kGMaxSlots, kGAbort = 16 * kGMaxSlots,
                   kGTokS = kGAbort + 16, kGSlotS = kGTokS + 4 * kGTok, kGFixedEnd = 384;
static_assert(kGSlotS + 4 * kGTok <= kGFixedEnd, "fixed map");

// Correction term of one group for NB blocks: acc += s * (D - (P + z Q)), the scale
// and zero point read once for all blocks; gs[nb] = (P, Q) of tokens 2t and 2t + 1.
template <typename S, int NB>
DEVI void flush_nb(float (&acc)[NB][4], const float (&d0)[NB][4], const float (&d1)[NB][4], const uint8_t* rec,
                   const TileGeom& tg, int grp, int g, const float4 (&gs)[NB]) {
  const uint32_t zz = tg.has_zeros ? (uint32_t)rec[tg.off_zero + grp * 8 + g] : 0x88u;
  const float za = (float)(zz & 15u), zb = (float)(zz >> 4);
  const float2 s = scale_pair(reinterpret_cast<const uint32_t*>(rec + tg.off_scale)[grp * 8 + g], (S*)nullptr);
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    acc[nb][0] = fmaf(s.x, (d0[nb][0] + d1[nb][0]) - fmaf(za, gs[nb].y, gs[nb].x), acc[nb][0]);
    acc[nb][1] = fmaf(s.x, (d0[nb][1] + d1[nb][1]) - fmaf(za, gs[nb].w, gs[nb].z), acc[nb][1]);
    acc[nb][2] = fmaf(s.y, (d0[nb][2] + d1[nb][2]) - fmaf(zb, gs[nb].y, gs[nb].x), acc[nb][2]);
    acc[nb][3] = fmaf(s.y, (d0[nb][3] + d1[nb][3]) - fmaf(zb, gs[nb].w, gs[nb].z), acc[nb][3]);
  }
}

// One pair's weights against NB blocks of staged rows (xp: this lane's row g of block
// 0 at the pair; blocks 8 rows apart).  With one block the MMAs alternate between two
// accumulator chains (k-steps A and B of each 32-column window) so that consecutive
// MMAs do not wait on each other; with two or three blocks the blocks are the
// independent chains (d1 stays unused, flush_nb adds its zeros).
// FIRST: the group's first pair (C = 0).
template <typename T, int NB, bool FIRST>
DEVI void pair_mma(float (&d0)[NB][4], float (&d1)[NB][4], uint4 w, const uint8_t* xp, uint32_t pitch8) {
  uint32_t A0[4], B0[4], A1[4], B1[4];
  DqOff<T>::expand(w.x, w.y, A0, B0);
  DqOff<T>::expand(w.z, w.w, A1, B1);
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const uint4 xa = *reinterpret_cast<const uint4*>(xp + nb * pitch8);
    const uint4 xb = *reinterpret_cast<const uint4*>(xp + nb * pitch8 + 64);
    float (&db)[4] = NB == 1 ? d1[nb] : d0[nb];
    if (FIRST) {
      mma_first<T>(d0[nb], A0[0], A0[1], A0[2], A0[3], xa.x, xa.y);
      if (NB == 1)
        mma_first<T>(db, B0[0], B0[1], B0[2], B0[3], xa.z, xa.w);
      else
        MmaOp<T>::run(db, B0[0], B0[1], B0[2], B0[3], xa.z, xa.w);
    } else {
      MmaOp<T>::run(d0[nb], A0[0], A0[1], A0[2], A0[3], xa.x, xa.y);
      MmaOp<T>::run(db, B0[0], B0[1], B0[2], B0[3], xa.z, xa.w);
    }
    MmaOp<T>::run(d0[nb], A1[0], A1[1], A1[2], A1[3], xb.x, xb.y);
    MmaOp<T>::run(db, B1[0], B1[1], B1[2], B1[3], xb.z, xb.w);
  }
}

// Fixed geometry: NPW pairs from pair pb, whole groups of PPG pairs, fully unrolled.
// gsg: per-group correction sums [group][kGPad].
template <typename T, typename S, int NB, int NPW, int PPG>
DEVI void gmm_fixed(const uint8_t* rec, const TileGeom& tg, int pb, int lane, const uint8_t* xsh,
                    uint32_t pitch, const float2* gsg, float (&acc)[NB][4]) {
  static_assert(NPW % PPG == 0, "warp ranges must hold whole groups");
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* wp = rec + (((uint32_t)pb << 5) + lane) * 16u;
  const uint8_t* xp = xsh + (uint32_t)g * pitch + (uint32_t)t * 16u + (uint32_t)pb * 128u;
  const uint32_t pitch8 = pitch * 8u;
#pragma unroll
  for (int gi = 0; gi < NPW / PPG; ++gi) {
    float d0[NB][4], d1[NB][4];
    if (NB > 1) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) zero4(d1[nb]);
    }
#pragma unroll
    for (int k = 0; k < PPG; ++k) {
      const int pi = gi * PPG + k;
      const uint4 w = *reinterpret_cast<const uint4*>(wp + pi * 512);
      if (k == 0)
        pair_mma<T, NB, true>(d0, d1, w, xp + pi * 128, pitch8);
      else
        pair_mma<T, NB, false>(d0, d1, w, xp + pi * 128, pitch8);
    }
    const int grp = pb / PPG + gi;
    float4 gs[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) gs[nb] = *reinterpret_cast<const float4*>(gsg + grp * kGPad + nb * 8 + 2 * t);
    flush_nb<S, NB>(acc, d0, d1, rec, tg, grp, g, gs);
  }
}

// Any geometry: pairs [pb, pe), groups cut where they begin and end, per-pair sums
// gx [pair][kGPad] accumulated over the pairs of a group this warp covers.
template <typename T, typename S, int NB>
DEVI void gmm_pairs(const uint8_t* rec, const TileGeom& tg, int pb, int pe, int lane, const uint8_t* xsh,
                    uint32_t pitch, const float2* gx, float (&acc)[NB][4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint32_t pitch8 = pitch * 8u;
  const uint8_t* xrow = xsh + (uint32_t)g * pitch + (uint32_t)t * 16u;
  int p = pb;
  while (p < pe) {
    const int grp = p >> tg.gshift;
    int pend = (grp + 1) << tg.gshift;
    if (pend > pe) pend = pe;
    float d0[NB][4], d1[NB][4];
    if (NB > 1) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) zero4(d1[nb]);
    }
    float4 gs[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) gs[nb] = make_float4(0.f, 0.f, 0.f, 0.f);
    bool first = true;
    for (; p < pend; ++p) {
      const uint4 w = *reinterpret_cast<const uint4*>(rec + (((uint32_t)p << 5) + lane) * 16u);
      if (first)
        pair_mma<T, NB, true>(d0, d1, w, xrow + (uint32_t)p * 128u, pitch8);
      else
        pair_mma<T, NB, false>(d0, d1, w, xrow + (uint32_t)p * 128u, pitch8);
      first = false;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const float4 gq = *reinterpret_cast<const float4*>(gx + p * kGPad + nb * 8 + 2 * t);
        gs[nb].x += gq.x;
        gs[nb].y += gq.y;
        gs[nb].z += gq.z;
        gs[nb].w += gq.w;
      }
    }
    flush_nb<S, NB>(acc, d0, d1, rec, tg, grp, g, gs);
  }
}

// Partial sums of lane (g, t) -> red[warp][nb][q][lane]; read back per (row, token).
template <int NB>
DEVI void put_acc(float* red, int warp, int lane, const float (&acc)[NB][4]) {
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) red[((warp * NB + nb) * 4 + q) * 32 + lane] = acc[nb][q];
}

// index of (row, token) in warp 0's partials; warp w's is this + w * NB * 128
template <int NB>
DEVI int acc_at0(int row, int tok) {
  const int g = row & 7, q = (row >> 3) * 2 + (tok & 1), t = (tok & 7) >> 1, nb = tok >> 3;
  return (nb * 4 + q) * 32 + g * 4 + t;
}

// Correction sums (P, Q) of 8 fragment-ordered 16-bit values (odd columns of fp16 rows
// already scaled by 1/16): se over the even columns, so over the odd ones.
template <typename T>
DEVI void frag_sums(const uint4& o, float& se, float& so) {
  const T* v = reinterpret_cast<const T*>(&o);
  se += (to_f32<T>(v[0]) + to_f32<T>(v[1])) + (to_f32<T>(v[4]) + to_f32<T>(v[5]));
  so += (to_f32<T>(v[2]) + to_f32<T>(v[3])) + (to_f32<T>(v[6]) + to_f32<T>(v[7]));
}

template <typename T>
DEVI float2 corr_pq(float se, float so) {
  const float P = DqOff<T>::kOddDiv16 ? 1024.f * (se + so) : 128.f * (se + so);
  const float Q = DqOff<T>::kOddDiv16 ? fmaf(16.f, so, se) : se + so;
  return make_float2(P, Q);
}

// per-group sums from the per-pair table, in pair order
DEVI void group_sums(const float2* gx, float2* gxg, int ngroups, int ppg, int tid) {
  for (int idx = tid; idx < ngroups * kGPad; idx += kConsumers) {
    const int grp = idx / kGPad, tk = idx - grp * kGPad;
    float2 s = gx[(grp * ppg) * kGPad + tk];
    for (int k = 1; k < ppg; ++k) {
      const float2 v = gx[(grp * ppg + k) * kGPad + tk];
      s.x += v.x;
      s.y += v.y;
    }
    gxg[idx] = s;
  }
}

// The ring of one CTA: slot s, phase bit ph, both advanced once per stage by the
// producer and by the consumers alike.
struct GRing {
  int slot = 0;
  uint32_t ph = 0;
  int n = 0;  // stages so far
  DEVI void next(int ns) {
    ++n;
    if (++slot == ns) {
      slot = 0;
      ph ^= 1u;
    }
  }
};

// Producer: arm slot r.slot for `bytes` and issue the copy, after the consumers
// released the slot's previous use.  Returns false (nothing issued) after an abort.
DEVI bool g_issue(uint64_t* full, uint64_t* empty, volatile int* abort_flag, int* err, const GRing& r, int ns,
                  uint8_t* dst, const uint8_t* src, uint32_t bytes, uint64_t pol) {
  if (*abort_flag) return false;
  if (r.n >= ns) {
    const long long t0 = clock64();
    while (!mbar_try_wait(&empty[r.slot], r.ph ^ 1u)) {
      if (*abort_flag) return false;
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort_flag = 1;
        set_error(err, DUPLEX_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
  mbar_arrive_expect_tx(&full[r.slot], bytes);
  bulk_g2s_stream(dst, src, bytes, &full[r.slot], pol);
  return true;
}

// Producer exit: wait (bounded) for the last min(n, ns) issued copies.
DEVI void g_drain(uint64_t* full, int n, int ns, int* err) {
  for (int j = n > ns ? n - ns : 0; j < n; ++j) {
    const long long t0 = clock64();
    while (!mbar_try_wait(&full[j % ns], (uint32_t)(j / ns) & 1u))
      if (clock64() - t0 > 200000000LL) {
        set_error(err, DUPLEX_DEVERR_TIMEOUT);
        break;
      }
  }
}

DEVI void g_range(int W, int& i0, int& i1) {
  i0 = (int)((long long)W * blockIdx.x / gridDim.x);
  i1 = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
}

DEVI void g_init(uint64_t* full, uint64_t* empty, volatile int* abort_flag, int ns, int consumers_per_stage) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], consumers_per_stage);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
}

DEVI void g_unit(const GExpParams& p, int u, int& e, int& first, int& n) {
  e = p.units[u * 3 + 0];
  e = (e < 0 || e >= p.E) ? 0 : e;
  first = p.units[u * 3 + 1];
  n = p.units[u * 3 + 2];
  n = n < 1 ? 1 : (n > p.tcap ? p.tcap : n);
}

// Ring position of the j-th stage of a CTA's range.
DEVI void g_slot(int j, int ns, int& slot, uint32_t& ph) {
  const int k = j / ns;
  slot = j - k * ns;
  ph = (uint32_t)k & 1u;
}

// Consumer wait for stage j (slot, phase ph) when the two warp groups take alternate
// stages: a slot's previous stage may belong to the other group, which may not have
// consumed it yet, and a parity wait on `full` that ran two phases ahead would return
// at once.  So first the release of stage j - ns (empty phase k - 1, k = j / ns): its
// phase k - 2 is complete (stage j - 2 ns is this group's own earlier stage, or came
// before the last re-staging barrier), so that wait cannot alias; once it passes,
// `full` is in the phase of stage j.
DEVI void g_wait_stage(uint64_t* full, uint64_t* empty, volatile int* abort_flag, int* err, int j, int ns,
                       int slot, uint32_t ph) {
  if (*abort_flag) return;
  const long long t0 = clock64();
  if (j >= ns) {
    while (!mbar_try_wait(&empty[slot], ph ^ 1u)) {
      if (*abort_flag) return;
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort_flag = 1;
        set_error(err, DUPLEX_DEVERR_TIMEOUT);
        return;
      }
    }
  }
  while (!mbar_try_wait(&full[slot], ph)) {
    if (*abort_flag) return;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      set_error(err, DUPLEX_DEVERR_TIMEOUT);
      return;
    }
  }
}

// Producer of both expert kernels: stages i0 .. i1-1 of the flattened list, stage
// `it` = (unit it / per_unit, part it % per_unit) at src(e, part), bytes(part).
template <typename Src>
DEVI void g_produce(const GExpParams& p, uint64_t* full, uint64_t* empty, volatile int* abort_flag,
                    uint8_t* ring, uint32_t slot_bytes, int ns, int i0, int i1, int per_unit, Src src) {
  const uint64_t pol = policy_evict_first();
  GRing r;
  for (int it = i0; it < i1; ++it) {
    const int u = it / per_unit, part = it - u * per_unit;
    int e, first, n;
    g_unit(p, u, e, first, n);
    uint32_t bytes;
    const uint8_t* from = src(e, part, bytes);
    if (!g_issue(full, empty, abort_flag, p.err, r, ns, ring + (uint32_t)r.slot * slot_bytes, from, bytes, pol))
      break;
    r.next(ns);
  }
  g_drain(full, r.n, ns, p.err);
}

// ---- gate|up item of one 8-warp group: warps 0-3 the gate record, 4-7 the up record,
// 4-way K split; act[first + tk][rb*16 .. +16] = SiLU(gate) * up.  red: this group's
// partials [8 warps][NB][4][32]; bar: the group's named barrier (256 threads).
// The tile geometry and pitches come in by value (copied once per kernel into
// registers): read through the parameter block, the compiler reloads them after every
// shared-memory store it cannot tell apart from that block, inside the pair loop.
template <typename T, typename S, int NB, int NPW, int PPG>
DEVI void gu_item(const TileGeom tg, uint32_t x_pitch, uint8_t* act, int I, const uint8_t* st,
                  uint64_t* empty_slot, int rb, int first, int n, const uint8_t* xsh, const float2* gx,
                  const float2* gxg, float* red, int bar) {
  const int lane = threadIdx.x & 31, wi = (threadIdx.x >> 5) & 7, gt = threadIdx.x & 255;
  const int rec = wi >> 2, kq = wi & 3;
  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) zero4(acc[nb]);
  const uint8_t* rp = st + (uint32_t)rec * tg.rec_bytes;
  if constexpr (NPW > 0) {
    gmm_fixed<T, S, NB, NPW, PPG>(rp, tg, kq * NPW, lane, xsh, x_pitch, gxg, acc);
  } else {
    const int np = tg.npairs;
    gmm_pairs<T, S, NB>(rp, tg, (kq * np) >> 2, ((kq + 1) * np) >> 2, lane, xsh, x_pitch, gx, acc);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_slot);
  put_acc<NB>(red, wi, lane, acc);
  named_bar_sync(bar, 256);
  constexpr int WS = NB * 128;  // one warp's partials
  for (int o = gt; o < 16 * n; o += 256) {
    const int row = o & 15, tk = o >> 4;
    const float* rr = red + acc_at0<NB>(row, tk);
    const float gsum_ = (rr[0] + rr[WS]) + (rr[2 * WS] + rr[3 * WS]);
    const float usum = (rr[4 * WS] + rr[5 * WS]) + (rr[6 * WS] + rr[7 * WS]);
    const int col = rb * 16 + row;
    T a = from_f32<T>(silu_f32(gsum_) * usum);
    if (DqOff<T>::kOddDiv16 && (col & 1)) a = from_f32<T>(to_f32<T>(a) * 0.0625f);
    reinterpret_cast<T*>(act + (size_t)(first + tk) * I * 2)[frag_pos(col)] = a;
  }
  named_bar_sync(bar, 256);
}

// Unit segments of a CTA's range: [it, seg_end) all belong to unit it / per_unit.
DEVI int g_seg_end(int it, int i1, int per_unit) {
  const int e = (it / per_unit + 1) * per_unit;
  return e < i1 ? e : i1;
}

template <typename T, typename S, int NPW, int PPG>
__global__ void __launch_bounds__(kThreads, 1) g_gateup_kernel(const __grid_constant__ GExpParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kGEmpty);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kGAbort);
  int* tok = reinterpret_cast<int*>(smem + kGTokS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int perG = p.I >> 4, ns = p.ns_a;
  pdl_launch_dependents();
  g_init(full, empty, abort_flag, ns, kCW / 2);
  pdl_wait();  // the unit list and tokens come from the previous launches
  int nu = *p.n_units;
  nu = nu < 0 ? 0 : (nu > p.max_units ? p.max_units : nu);
  int i0, i1;
  g_range(nu * perG, i0, i1);
  uint8_t* ring = smem + p.off_ring_a;

  if (warp == kCW) {
    if (lane != 0) return;
    g_produce(p, full, empty, abort_flag, ring, p.slot_a, ns, i0, i1, perG,
              [&](int e, int rb, uint32_t& bytes) {
                bytes = 2u * p.tgu.rec_bytes;
                return p.gu_tiles + ((size_t)e * 2 * perG + 2 * rb) * p.tgu.rec_bytes;
              });
    return;
  }

  uint8_t* xsh = smem + p.off_x;
  float2* gx = reinterpret_cast<float2*>(smem + p.off_gx);
  float2* gxg = reinterpret_cast<float2*>(smem + p.off_gxg);
  const TileGeom tgu = p.tgu;
  const uint32_t x_pitch = p.x_pitch;
  uint8_t* const act = p.act;
  const int I = p.I;
  const int grp = warp >> 3;
  float* red = reinterpret_cast<float*>(smem + p.off_red_a) + grp * p.red_floats;
  const int H = p.H, np = p.tgu.npairs;
  for (int s0 = i0; s0 < i1;) {
    const int s1 = g_seg_end(s0, i1, perG);
    // ---- the unit's token rows in fragment order (fp16: odd columns / 16) and their
    // correction sums per pair and per group (zero for absent tokens)
    int e, first, n;
    g_unit(p, s0 / perG, e, first, n);
    named_bar_sync(1, kConsumers);  // both groups are done with the previous unit
    if (tid < n) tok[tid] = p.assign[first + tid] >> 3;
    named_bar_sync(1, kConsumers);
    // a thread's row loads are issued kRL at a time before any is used (one memory
    // latency per kRL passes)
    const int nq = H >> 3, total = n * nq;
    constexpr int kRL = 5;  // loads in flight per thread (two rounds for 20 tokens at hidden 2048)
    for (int base0 = 0; base0 < total; base0 += kRL * kConsumers) {
      uint4 ld[kRL];
#pragma unroll
      for (int k = 0; k < kRL; ++k) {
        const int idx = base0 + k * kConsumers + tid;
        if (idx < total) {
          const int rr = idx / nq, q = idx - rr * nq;
          ld[k] = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)tok[rr] * p.x_row_bytes) + q);
        }
      }
#pragma unroll
      for (int k = 0; k < kRL; ++k) {
      const int idx = base0 + k * kConsumers + tid;
      float se = 0.f, so = 0.f;
      int rr = 0, q = 0;
      if (idx < total) {
        rr = idx / nq;
        q = idx - rr * nq;
        uint4 o = to_frag_order(ld[k]);
        if (DqOff<T>::kOddDiv16) {
          const __half2 q16 = __float2half2_rn(0.0625f);
          __half2 hy = __hmul2(*reinterpret_cast<__half2*>(&o.y), q16);
          __half2 hw = __hmul2(*reinterpret_cast<__half2*>(&o.w), q16);
          o.y = *reinterpret_cast<uint32_t*>(&hy);
          o.w = *reinterpret_cast<uint32_t*>(&hw);
        }
        *reinterpret_cast<uint4*>(xsh + (uint32_t)rr * p.x_pitch + (uint32_t)q * 16u) = o;
        frag_sums<T>(o, se, so);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        so += __shfl_xor_sync(0xffffffffu, so, o);
      }
      if (idx < total && (q & 7) == 0) gx[(q >> 3) * kGPad + rr] = corr_pq<T>(se, so);
      }
    }
    for (int idx = tid; idx < np * kGPad; idx += kConsumers)
      if (idx % kGPad >= n) gx[idx] = make_float2(0.f, 0.f);
    named_bar_sync(1, kConsumers);
    group_sums(gx, gxg, np >> p.tgu.gshift, 1 << p.tgu.gshift, tid);
    named_bar_sync(1, kConsumers);
    // ---- the segment's items, alternately to the two groups
    const int nbv = (n + 7) >> 3;
    for (int it = s0 + grp; it < s1; it += 2) {
      int slot;
      uint32_t ph;
      g_slot(it - i0, ns, slot, ph);
      g_wait_stage(full, empty, abort_flag, p.err, it - i0, ns, slot, ph);
      const uint8_t* st = ring + (uint32_t)slot * p.slot_a;
      const int rb = it - (it / perG) * perG;
      if (nbv == 1)
        gu_item<T, S, 1, NPW, PPG>(tgu, x_pitch, act, I, st, &empty[slot], rb, first, n, xsh, gx, gxg, red,
                                   2 + grp);
      else if (nbv == 2)
        gu_item<T, S, 2, NPW, PPG>(tgu, x_pitch, act, I, st, &empty[slot], rb, first, n, xsh, gx, gxg, red,
                                   2 + grp);
      else
        gu_item<T, S, 3, NPW, PPG>(tgu, x_pitch, act, I, st, &empty[slot], rb, first, n, xsh, gx, gxg, red,
                                   2 + grp);
    }
    s0 = s1;
  }
}

// ---- down item: one warp, one record (16 rows of H) over the whole K; the outputs
// go from the accumulators straight to ypart[tok][slot][row] for the live tokens.
template <typename T, typename S, int NB, int NPW, int PPG>
DEVI void dn_item(const TileGeom tg, uint32_t a_pitch, float* ypart, int top_k, int H, const uint8_t* rp,
                  uint64_t* empty_slot, int row0, int n, const int* tok, const int* slt, const uint8_t* act,
                  const float2* ga, const float2* gag) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) zero4(acc[nb]);
  if (rp) {
    if constexpr (NPW > 0)
      gmm_fixed<T, S, NB, NPW, PPG>(rp, tg, 0, lane, act, a_pitch, gag, acc);
    else
      gmm_pairs<T, S, NB>(rp, tg, 0, tg.npairs, lane, act, a_pitch, ga, acc);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_slot);
  if (!rp) return;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int tk = nb * 8 + 2 * t + (q & 1), row = row0 + g + (q >> 1) * 8;
      if (tk < n) ypart[((size_t)tok[tk] * top_k + slt[tk]) * H + row] = acc[nb][q];
    }
}

template <typename T, typename S, int NPW, int PPG>
__global__ void __launch_bounds__(kThreads, 1) g_down_kernel(const __grid_constant__ GExpParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kGEmpty);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kGAbort);
  int* tok = reinterpret_cast<int*>(smem + kGTokS);
  int* slt = reinterpret_cast<int*>(smem + kGSlotS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int RbD = p.H >> 4, nDN = (RbD + kGDnRec - 1) / kGDnRec, ns = p.ns_d;
  pdl_launch_dependents();
  g_init(full, empty, abort_flag, ns, kCW / 2);
  pdl_wait();  // the unit list and tokens come from the previous launches
  int nu = *p.n_units;
  nu = nu < 0 ? 0 : (nu > p.max_units ? p.max_units : nu);
  int i0, i1;
  g_range(nu * nDN, i0, i1);
  uint8_t* ring = smem + p.off_ring_d;

  if (warp == kCW) {
    if (lane != 0) return;
    g_produce(p, full, empty, abort_flag, ring, p.slot_d, ns, i0, i1, nDN,
              [&](int e, int s, uint32_t& bytes) {
                const int cnt = RbD - kGDnRec * s < kGDnRec ? RbD - kGDnRec * s : kGDnRec;
                bytes = (uint32_t)cnt * p.tdn.rec_bytes;
                return p.dn_tiles + ((size_t)e * RbD + kGDnRec * s) * p.tdn.rec_bytes;
              });
    return;
  }

  uint8_t* act = smem + p.off_a;
  float2* ga = reinterpret_cast<float2*>(smem + p.off_ga);
  float2* gag = reinterpret_cast<float2*>(smem + p.off_gag);
  const TileGeom tdn = p.tdn;
  const uint32_t a_pitch = p.a_pitch;
  float* const ypart = p.ypart;
  const int top_k = p.top_k, H = p.H;
  const int I = p.I, np = p.tdn.npairs;
  const int grp = warp >> 3, rc = warp & 7;
  for (int s0 = i0; s0 < i1;) {
    const int s1 = g_seg_end(s0, i1, nDN);
    // ---- the unit's intermediate rows (already in fragment order) and their
    // correction sums per pair and per group
    int e, first, n;
    g_unit(p, s0 / nDN, e, first, n);
    named_bar_sync(1, kConsumers);
    if (tid < n) {
      const int a = p.assign[first + tid];
      tok[tid] = a >> 3;
      slt[tid] = a & 7;
    }
    const int nq = I >> 3;
    for (int base0 = 0; base0 < n * nq; base0 += 4 * kConsumers) {
      uint4 ld[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = base0 + k * kConsumers + tid;
        if (idx < n * nq) {
          const int rr = idx / nq, q = idx - rr * nq;
          ld[k] = __ldcg(reinterpret_cast<const uint4*>(p.act + (size_t)(first + rr) * I * 2) + q);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = base0 + k * kConsumers + tid;
        if (idx < n * nq) {
          const int rr = idx / nq, q = idx - rr * nq;
          *reinterpret_cast<uint4*>(act + (uint32_t)rr * a_pitch + (uint32_t)q * 16u) = ld[k];
        }
      }
    }
    named_bar_sync(1, kConsumers);
    for (int idx = tid; idx < np * kGPad; idx += kConsumers) {
      const int pp = idx / kGPad, tk = idx - pp * kGPad;
      float se = 0.f, so = 0.f;
      if (tk < n) {
        const uint8_t* rowp = act + (uint32_t)tk * p.a_pitch + (uint32_t)pp * 128u;
#pragma unroll
        for (int c = 0; c < 8; ++c) frag_sums<T>(*reinterpret_cast<const uint4*>(rowp + c * 16), se, so);
      }
      ga[idx] = corr_pq<T>(se, so);
    }
    named_bar_sync(1, kConsumers);
    group_sums(ga, gag, np >> p.tdn.gshift, 1 << p.tdn.gshift, tid);
    named_bar_sync(1, kConsumers);
    // ---- the segment's stages, alternately to the two groups, one record per warp
    const int nbv = (n + 7) >> 3;
    for (int it = s0 + grp; it < s1; it += 2) {
      int slot;
      uint32_t ph;
      g_slot(it - i0, ns, slot, ph);
      g_wait_stage(full, empty, abort_flag, p.err, it - i0, ns, slot, ph);
      const int s = it - (it / nDN) * nDN;
      const int cnt = RbD - kGDnRec * s < kGDnRec ? RbD - kGDnRec * s : kGDnRec;
      const uint8_t* rp = rc < cnt ? ring + (uint32_t)slot * p.slot_d + (uint32_t)rc * p.tdn.rec_bytes : nullptr;
      const int row0 = (kGDnRec * s + rc) * 16;
      if (nbv == 1)
        dn_item<T, S, 1, NPW, PPG>(tdn, a_pitch, ypart, top_k, H, rp, &empty[slot], row0, n, tok, slt, act,
                                   ga, gag);
      else if (nbv == 2)
        dn_item<T, S, 2, NPW, PPG>(tdn, a_pitch, ypart, top_k, H, rp, &empty[slot], row0, n, tok, slt, act,
                                   ga, gag);
      else
        dn_item<T, S, 3, NPW, PPG>(tdn, a_pitch, ypart, top_k, H, rp, &empty[slot], row0, n, tok, slt, act,
                                   ga, gag);
    }
    s0 = s1;
  }
}

// ------------------------------------------------------------------ 5. combine
// out[t][r] = sum over the slots j in selection order whose expert is in
// [e_begin, e_begin + E) of w[t][j] * y[t][j][r] (+ residual[t][r]), rounded once to
// the output type O (the activation type, or fp32 partial sums for expert-parallel
// ranks); four consecutive outputs per thread.
template <typename T, typename O>
__global__ void __launch_bounds__(256) g_combine_kernel(const float* ypart, const float* w, const int* sel,
                                                        int meta_stride, int e_begin, int E, const T* residual,
                                                        int nT, int H, int top_k, O* out) {
  const int H4 = H >> 2;
  const size_t idx = (size_t)blockIdx.x * 256 + threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  if (idx >= (size_t)nT * H4) return;
  const int t = (int)(idx / H4), r4 = (int)(idx - (size_t)t * H4);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < top_k; ++j) {
    const unsigned e = (unsigned)(sel[(size_t)t * meta_stride + j] - e_begin);
    if (e >= (unsigned)E) continue;
    const float wj = w[(size_t)t * meta_stride + j];
    const float4 v = __ldcg(reinterpret_cast<const float4*>(ypart + ((size_t)t * top_k + j) * H) + r4);
    s.x = fmaf(wj, v.x, s.x);
    s.y = fmaf(wj, v.y, s.y);
    s.z = fmaf(wj, v.z, s.z);
    s.w = fmaf(wj, v.w, s.w);
  }
  const size_t o = (size_t)t * H + (size_t)r4 * 4;
  if (residual) {
    const uint2 rv = *reinterpret_cast<const uint2*>(residual + o);
    const T* rr = reinterpret_cast<const T*>(&rv);
    s.x += to_f32<T>(rr[0]);
    s.y += to_f32<T>(rr[1]);
    s.z += to_f32<T>(rr[2]);
    s.w += to_f32<T>(rr[3]);
  }
  if constexpr (std::is_same<O, float>::value) {
    *reinterpret_cast<float4*>(out + o) = s;
  } else {
    uint2 ov;
    O* oo = reinterpret_cast<O*>(&ov);
    oo[0] = from_f32<O>(s.x);
    oo[1] = from_f32<O>(s.y);
    oo[2] = from_f32<O>(s.z);
    oo[3] = from_f32<O>(s.w);
    *reinterpret_cast<uint2*>(out + o) = ov;
  }
}

// ====================================================================== host side
struct GScratch {
  size_t logits, sel, w, assign, units, n_units, act, ypart, total;
  int max_units;
};

// Unit token cap of one call, from the expected tokens per expert mu = T k / E: small
// batches stage fewer rows, which leaves room for a deeper weight ring.
static int g_tcap(int T, int E, int top_k) {
  const int tk = T * top_k;
  if (tk <= 4 * E) return 8;
  if (tk <= 9 * E) return 16;
  return kGTok;
}

static GScratch g_scratch(int T, int E, int H, int I, int top_k, int tcap) {
  GScratch s;
  size_t off = 0;
  s.max_units = E + (T * top_k + tcap - 1) / tcap + 1;
  s.logits = off; off += align_up((size_t)T * E * 4, 256);
  s.sel = off; off += align_up((size_t)T * top_k * 4, 256);
  s.w = off; off += align_up((size_t)T * top_k * 4, 256);
  s.assign = off; off += align_up((size_t)T * top_k * 4, 256);
  s.units = off; off += align_up((size_t)s.max_units * 12, 256);
  s.n_units = off; off += 256;
  s.act = off; off += align_up((size_t)T * top_k * I * 2, 256);
  s.ypart = off; off += align_up((size_t)T * top_k * H * 4, 256);
  s.total = off;
  return s;
}

// Shared-memory maps of the two expert kernels for one geometry and unit cap tcap (the
// ring takes what is left, up to kGMaxSlots slots, at least 2); false when a map does
// not fit.  The staged rows are sized for tcap tokens; MMA blocks read up to
// 8 ceil(tcap / 8) <= kGPad rows, which stay inside the map because the tables,
// partials and ring follow them.
static bool g_layout(int H, int I, int group, int has_zeros, int tcap, GExpParams* p) {
  if ((H & 63) || (I & 63) || group < 64 || (group & (group - 1))) return false;
  if (g_router_smem(H) > kGSmemMax) return false;  // router tile
  if (tile_geom(H, group, has_zeros, &p->tgu) || tile_geom(I, group, has_zeros, &p->tdn)) return false;
  auto up = [](uint32_t v, uint32_t a) { return (v + a - 1) / a * a; };
  p->x_pitch = up((uint32_t)H * 2u, 128) + 64u;
  p->a_pitch = up((uint32_t)I * 2u, 128) + 64u;
  const uint32_t ppg = 1u << p->tgu.gshift;
  p->tcap = tcap;
  p->red_floats = 8 * ((tcap + 7) / 8) * 128;
  // gate|up
  p->slot_a = up(2u * p->tgu.rec_bytes, 128);
  p->off_x = kGFixedEnd;
  p->off_gx = up(p->off_x + (uint32_t)tcap * p->x_pitch, 128);
  p->off_gxg = up(p->off_gx + (uint32_t)p->tgu.npairs * kGPad * 8u, 128);
  p->off_red_a = up(p->off_gxg + (uint32_t)p->tgu.npairs / ppg * kGPad * 8u, 128);
  p->off_ring_a = up(p->off_red_a + 2u * (uint32_t)p->red_floats * 4u, 128);
  if (p->off_ring_a + 2 * p->slot_a > (uint32_t)kGSmemMax) return false;
  p->ns_a = (int)((kGSmemMax - p->off_ring_a) / p->slot_a);
  if (p->ns_a > kGMaxSlots) p->ns_a = kGMaxSlots;
  p->smem_a = p->off_ring_a + (uint32_t)p->ns_a * p->slot_a;
  if (p->off_x + 8u * ((tcap + 7) / 8) * p->x_pitch > p->smem_a) return false;
  // down
  p->slot_d = up((uint32_t)kGDnRec * p->tdn.rec_bytes, 128);
  p->off_a = kGFixedEnd;
  p->off_ga = up(p->off_a + (uint32_t)tcap * p->a_pitch, 128);
  p->off_gag = up(p->off_ga + (uint32_t)p->tdn.npairs * kGPad * 8u, 128);
  p->off_ring_d = up(p->off_gag + (uint32_t)p->tdn.npairs / ppg * kGPad * 8u, 128);
  if (p->off_ring_d + 2 * p->slot_d > (uint32_t)kGSmemMax) return false;
  p->ns_d = (int)((kGSmemMax - p->off_ring_d) / p->slot_d);
  if (p->ns_d > kGMaxSlots) p->ns_d = kGMaxSlots;
  p->smem_d = p->off_ring_d + (uint32_t)p->ns_d * p->slot_d;
  if (p->off_a + 8u * ((tcap + 7) / 8) * p->a_pitch > p->smem_d) return false;
  return true;
}

// Kernel instances: the fixed-geometry loop where a warp's pair range holds whole
// groups (gate|up: a quarter of a record's K, down: a whole record), else the general one.
template <typename T, typename S>
static void (*g_gateup_fn(const TileGeom& tg))(GExpParams) {
  const int ppg = 1 << tg.gshift;
  if (tg.npairs == 32) {  // K = 2048
    if (ppg == 1) return g_gateup_kernel<T, S, 8, 1>;
    if (ppg == 2) return g_gateup_kernel<T, S, 8, 2>;
    if (ppg == 4) return g_gateup_kernel<T, S, 8, 4>;
  }
  return g_gateup_kernel<T, S, 0, 1>;
}

template <typename T, typename S>
static void (*g_down_fn(const TileGeom& tg))(GExpParams) {
  const int ppg = 1 << tg.gshift;
  if (tg.npairs == 12) {  // K = 768
    if (ppg == 1) return g_down_kernel<T, S, 12, 1>;
    if (ppg == 2) return g_down_kernel<T, S, 12, 2>;
    if (ppg == 4) return g_down_kernel<T, S, 12, 4>;
  }
  return g_down_kernel<T, S, 0, 1>;
}

// Launch on `st`; with pdl the kernel may start while the previous one on the stream
// finishes (programmatic dependent launch): every kernel here calls griddepcontrol.wait
// before it reads anything the previous launch wrote.
template <typename... KArgs, typename... Args>
static int g_launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return record_cuda(cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...));
}

// Bucketing, the two expert kernels and the combine, for the assignments in sel [T][k]
// whose experts are [e_begin, e_begin + E) (tiles indexed from e_begin); out [T][H] in
// the activation type (out_f32 == 0) or fp32.
static int g_expert_stage(const void* x, size_t x_row_bytes, bool f16, int T, const int* sel, const float* w,
                          int meta_stride, int top_k, int e_begin,
                          int E, int E_total, int H, int I, const void* gu_tiles, const void* dn_tiles,
                          GExpParams& p, const GScratch& L, int tcap, uint8_t* ws, const void* residual, void* out,
                          int out_f32, int* err, cudaStream_t st, bool pdl_first) {
  int rc;
  {
    const int N = T * top_k, nch = (N + 31) / 32;
    const int smem = (int)(align_up((size_t)nch * E, 16) + align_up((size_t)nch * E * 2, 16) +
                           3 * kMaxExperts * 4 + 16 * 4 + (size_t)N * 4);
    if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(g_bucket_kernel), kGSmemMax))) return rc;
    if ((rc = g_launch(g_bucket_kernel, dim3(1), dim3(512), smem, st, pdl_first, sel, meta_stride, T, E, top_k, tcap,
                       e_begin,
                       E_total, reinterpret_cast<int*>(ws + L.assign), reinterpret_cast<int*>(ws + L.units),
                       reinterpret_cast<int*>(ws + L.n_units), L.max_units, err)))
      return rc;
  }
  p.H = H; p.I = I; p.E = E; p.top_k = top_k; p.max_units = L.max_units;
  p.x = reinterpret_cast<const uint8_t*>(x);
  p.x_row_bytes = x_row_bytes;
  p.gu_tiles = reinterpret_cast<const uint8_t*>(gu_tiles);
  p.dn_tiles = reinterpret_cast<const uint8_t*>(dn_tiles);
  p.assign = reinterpret_cast<const int*>(ws + L.assign);
  p.units = reinterpret_cast<const int*>(ws + L.units);
  p.n_units = reinterpret_cast<const int*>(ws + L.n_units);
  p.act = ws + L.act;
  p.ypart = reinterpret_cast<float*>(ws + L.ypart);
  p.err = err;
  {
    void (*ka)(GExpParams) = f16 ? g_gateup_fn<__half, __half>(p.tgu)
                                 : g_gateup_fn<__nv_bfloat16, __nv_bfloat16>(p.tgu);
    void (*kd)(GExpParams) = f16 ? g_down_fn<__half, __half>(p.tdn)
                                 : g_down_fn<__nv_bfloat16, __nv_bfloat16>(p.tdn);
    if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(ka), kGSmemMax))) return rc;
    if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(kd), kGSmemMax))) return rc;
    const int G = num_sms();
    if ((rc = g_launch(ka, dim3(G), dim3(kThreads), p.smem_a, st, true, p))) return rc;
    if ((rc = g_launch(kd, dim3(G), dim3(kThreads), p.smem_d, st, true, p))) return rc;
  }
  const float* yp = reinterpret_cast<const float*>(ws + L.ypart);
  const unsigned blocks = (unsigned)(((size_t)T * H / 4 + 255) / 256);
  const dim3 cg(blocks), cb(256);
  if (f16) {
    const __half* res = reinterpret_cast<const __half*>(residual);
    if (out_f32)
      return g_launch(g_combine_kernel<__half, float>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res, T, H,
                      top_k, reinterpret_cast<float*>(out));
    return g_launch(g_combine_kernel<__half, __half>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res, T, H, top_k,
                    reinterpret_cast<__half*>(out));
  }
  const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(residual);
  if (out_f32)
    return g_launch(g_combine_kernel<__nv_bfloat16, float>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res, T, H,
                    top_k, reinterpret_cast<float*>(out));
  return g_launch(g_combine_kernel<__nv_bfloat16, __nv_bfloat16>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res,
                  T, H, top_k, reinterpret_cast<__nv_bfloat16*>(out));
}

// Router logits (unless given) and top-k: sel / w [T][top_k] (and the optional copies
// sel_out / w_out, and the exchange rows in pack).
static int g_route(const void* x, bool f16, int T, const void* gate_w, const void* gate_b, const float* logits_in,
                   int E, int H, int top_k, int norm_topk, uint8_t* ws, const GScratch& L, int* sel, float* w,
                   int32_t* sel_out, float* w_out, uint8_t* pack, int64_t pack_row, int* err, cudaStream_t st) {
  int rc;
  float* logits = logits_in ? const_cast<float*>(logits_in) : reinterpret_cast<float*>(ws + L.logits);
  // router
  if (!logits_in) {
    const int smem = g_router_smem(H);
    void (*rk)(const __half*, const __half*, const __half*, int, int, int, float*, int*) = g_router_kernel<__half>;
    void (*rkb)(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, int, int, int, float*, int*) =
        g_router_kernel<__nv_bfloat16>;
    const void* fn = f16 ? reinterpret_cast<const void*>(rk) : reinterpret_cast<const void*>(rkb);
    // the attribute is set once per kernel (to the ceiling), whatever this call's size
    if (smem > kGSmemMax) return DUPLEX_ERR_UNSUPPORTED;
    if ((rc = ensure_smem_attr(fn, kGSmemMax))) return rc;
    const dim3 grid((E + 15) / 16, (T + 15) / 16);
    if (f16)
      rc = g_launch(rk, grid, dim3(256), smem, st, false, reinterpret_cast<const __half*>(x),
                    reinterpret_cast<const __half*>(gate_w), reinterpret_cast<const __half*>(gate_b), T, E, H, logits,
                    err);
    else
      rc = g_launch(rkb, grid, dim3(256), smem, st, false, reinterpret_cast<const __nv_bfloat16*>(x),
                    reinterpret_cast<const __nv_bfloat16*>(gate_w), reinterpret_cast<const __nv_bfloat16*>(gate_b),
                    T, E, H, logits, err);
    if (rc) return rc;
  }
  // top-k
  const bool pdl = !logits_in;  // after the router launch
  const dim3 grid((T + 15) / 16), block(512);
  const float* lg = logits;
  if (f16) {
    const __half* xh = reinterpret_cast<const __half*>(x);
    return pack ? g_launch(g_topk_kernel<__half, true>, grid, block, 0, st, pdl, lg, T, E, top_k, norm_topk, sel, w,
                           sel_out, w_out, xh, H, pack, pack_row)
                : g_launch(g_topk_kernel<__half, false>, grid, block, 0, st, pdl, lg, T, E, top_k, norm_topk, sel, w,
                           sel_out, w_out, xh, H, pack, pack_row);
  }
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  return pack ? g_launch(g_topk_kernel<__nv_bfloat16, true>, grid, block, 0, st, pdl, lg, T, E, top_k, norm_topk, sel,
                         w, sel_out, w_out, xb, H, pack, pack_row)
              : g_launch(g_topk_kernel<__nv_bfloat16, false>, grid, block, 0, st, pdl, lg, T, E, top_k, norm_topk, sel,
                         w, sel_out, w_out, xb, H, pack, pack_row);
}

static bool g_misaligned(std::initializer_list<const void*> ptrs) {
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return true;
  return false;
}

}  // namespace duplex

#include "grouped_tc.cuh"

using namespace duplex;

extern "C" int duplex_moe_grouped_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                                  int32_t top_k, int32_t group, int has_zeros,
                                                  size_t* bytes) {
  if (!bytes || T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 ||
      top_k > kMaxTopK || top_k > E || H < 1 || I < 1)
    return DUPLEX_ERR_ARG;
  GExpParams p = {};
  if (!g_layout(H, I, group, has_zeros, kGTok, &p)) return DUPLEX_ERR_UNSUPPORTED;  // every cap fits
  *bytes = g_scratch(T, E, H, I, top_k, g_tcap(T, E, top_k)).total;
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
  if (!g_layout(H, I, group, has_zeros, kGTok, &p)) return DUPLEX_ERR_UNSUPPORTED;
  const int tcap = g_tcap(T, E, top_k);
  if (!g_layout(H, I, group, has_zeros, tcap, &p)) return DUPLEX_ERR_UNSUPPORTED;
  const GScratch L = g_scratch(T, E, H, I, top_k, tcap);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if (g_misaligned({x, out, workspace, gu_tiles, dn_tiles, gate_w, residual, logits_in})) return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  int* sel = reinterpret_cast<int*>(ws + L.sel);
  float* w = reinterpret_cast<float*>(ws + L.w);
  cudaStream_t st = (cudaStream_t)stream;
  const bool f16 = act_dtype == DUPLEX_DTYPE_F16;
  int rc;
  if ((rc = g_route(x, f16, T, gate_w, gate_b, logits_in, E, H, top_k, norm_topk, ws, L, sel, w, sel_out, w_out,
                    nullptr, 0, err, st)))
    return rc;
  // 3-5. bucketing, experts, combine
  return g_expert_stage(x, (size_t)H * 2, f16, T, sel, w, top_k, top_k, 0, E, E, H, I, gu_tiles, dn_tiles, p, L,
                        tcap, ws, residual, out, 0, err, st, true);
}

extern "C" int duplex_moe_experts_grouped_workspace_bytes(int32_t T, int32_t E_local, int32_t E_total,
                                                          int32_t H, int32_t I, int32_t top_k, int32_t group,
                                                          int has_zeros, size_t* bytes) {
  if (!bytes || T < 1 || T > kGMaxT || E_local < 1 || E_total < E_local || E_total > kMaxExperts ||
      top_k < 1 || top_k > kMaxTopK || top_k > E_total || H < 1 || I < 1)
    return DUPLEX_ERR_ARG;
  GExpParams p = {};
  if (!g_layout(H, I, group, has_zeros, kGTok, &p)) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = g_scratch(T, E_local, H, I, top_k, g_tcap(T, E_total, top_k)).total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_experts_grouped(const void* x, int act_dtype, int32_t T, int64_t x_row_stride,
                                          const int32_t* sel, const float* w, int32_t meta_stride, int32_t top_k,
                                          int32_t e_begin, int32_t E_local,
                                          int32_t E_total, int32_t H, int32_t I, const void* gu_tiles,
                                          const void* dn_tiles, int scale_dtype, int has_zeros, int32_t group,
                                          const void* residual, void* out, int out_dtype, void* workspace,
                                          size_t workspace_bytes, int32_t* err, void* stream) {
  if (!x || !sel || !w || !out || !gu_tiles || !dn_tiles || !workspace) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kGMaxT || E_local < 1 || e_begin < 0 || e_begin + E_local > E_total ||
      E_total > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E_total)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  if (out_dtype != act_dtype && out_dtype != DUPLEX_DTYPE_F32) return DUPLEX_ERR_DTYPE;
  GExpParams p = {};
  if (!g_layout(H, I, group, has_zeros, kGTok, &p)) return DUPLEX_ERR_UNSUPPORTED;
  const int tcap = g_tcap(T, E_total, top_k);
  if (!g_layout(H, I, group, has_zeros, tcap, &p)) return DUPLEX_ERR_UNSUPPORTED;
  const GScratch L = g_scratch(T, E_local, H, I, top_k, tcap);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  if (x_row_stride < H || (x_row_stride & 7)) return DUPLEX_ERR_ALIGN;
  if (meta_stride < top_k) return DUPLEX_ERR_ARG;
  if (g_misaligned({x, out, workspace, gu_tiles, dn_tiles, residual})) return DUPLEX_ERR_ALIGN;
  return g_expert_stage(x, (size_t)x_row_stride * 2, act_dtype == DUPLEX_DTYPE_F16, T, sel, w, meta_stride, top_k,
                        e_begin,
                        E_local, E_total, H, I,
                        gu_tiles, dn_tiles, p, L, tcap, reinterpret_cast<uint8_t*>(workspace), residual, out,
                        out_dtype == DUPLEX_DTYPE_F32, err, (cudaStream_t)stream, false);
}

extern "C" int duplex_moe_route_grouped(const void* x, int act_dtype, int32_t T, const void* gate_w,
                                        const void* gate_b, const float* logits_in, int32_t E, int32_t H,
                                        int32_t top_k, int32_t norm_topk, float* w_out, int32_t* sel_out,
                                        void* pack, int64_t pack_row_bytes, void* workspace,
                                        size_t workspace_bytes, int32_t* err, void* stream) {
  if (!x || !workspace || (!gate_w && !logits_in) || (!pack && (!w_out || !sel_out))) return DUPLEX_ERR_ARG;
  if (pack && (pack_row_bytes < (int64_t)H * 2 + 8 * top_k || (pack_row_bytes & 15) ||
               (reinterpret_cast<uintptr_t>(pack) & 15u)))
    return DUPLEX_ERR_ALIGN;
  if (T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (H < 8 || (H & 7)) return DUPLEX_ERR_UNSUPPORTED;
  if (g_router_smem(H) > kGSmemMax) return DUPLEX_ERR_UNSUPPORTED;
  const GScratch L = g_scratch(T, E, H, 64, top_k, 8);
  if (workspace_bytes < L.logits + (size_t)T * E * 4) return DUPLEX_ERR_WORKSPACE;
  if (g_misaligned({x, gate_w, logits_in, workspace})) return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  return g_route(x, act_dtype == DUPLEX_DTYPE_F16, T, gate_w, gate_b, logits_in, E, H, top_k, norm_topk, ws, L,
                 sel_out, w_out, nullptr, nullptr, reinterpret_cast<uint8_t*>(pack), pack_row_bytes, err,
                 (cudaStream_t)stream);
}

// ------------------------------------------------------------ tcgen05 expert path
extern "C" int duplex_tc_records_bytes(int32_t E, int32_t R, int32_t K, int32_t group, int has_zeros,
                                       int32_t pair_halves, size_t* bytes) {
  if (!bytes || E < 1 || R < 1 || K < 1) return DUPLEX_ERR_ARG;
  if (group != kTcK || K % kTcK || R % kTcM || (pair_halves && (R % 128))) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = (size_t)E * (R / kTcM) * (K / kTcK) * tc_chunk_bytes(has_zeros);
  return DUPLEX_OK;
}

extern "C" int duplex_repack_tc_records(const int32_t* packed, const void* scale, const int32_t* zeros,
                                        int scale_dtype, int32_t E, int32_t R, int32_t K, int32_t group,
                                        int32_t pair_halves, void* records, size_t records_bytes, void* stream) {
  if (!packed || !scale || !records) return DUPLEX_ERR_ARG;
  size_t need = 0;
  int rc = duplex_tc_records_bytes(E, R, K, group, zeros != nullptr, pair_halves, &need);
  if (rc) return rc;
  if (records_bytes < need) return DUPLEX_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(records) & 15u) return DUPLEX_ERR_ALIGN;
  const long long words = (long long)(need / 4);
  int blocks = (int)((words + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  cudaStream_t st = (cudaStream_t)stream;
  const uint32_t cb = tc_chunk_bytes(zeros != nullptr);
  if (scale_dtype == DUPLEX_DTYPE_F16)
    tc_repack_kernel<__half><<<blocks, 256, 0, st>>>(packed, reinterpret_cast<const __half*>(scale), zeros, E, R, K,
                                                     pair_halves, cb, reinterpret_cast<uint32_t*>(records));
  else if (scale_dtype == DUPLEX_DTYPE_BF16)
    tc_repack_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(packed, reinterpret_cast<const __nv_bfloat16*>(scale),
                                                            zeros, E, R, K, pair_halves, cb,
                                                            reinterpret_cast<uint32_t*>(records));
  else
    return DUPLEX_ERR_DTYPE;
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_moe_grouped_tc_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I, int32_t top_k,
                                                     int32_t group, int has_zeros, size_t* bytes) {
  (void)has_zeros;
  if (!bytes || T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E)
    return DUPLEX_ERR_ARG;
  if (!tc_geometry_ok(H, I, group) || g_router_smem(H) > kGSmemMax) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = tc_scratch(T, E, H, I, top_k, tc_cols(T, E, top_k)).g.total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_grouped_tc(const void* x, int act_dtype, int32_t T, const void* gate_w,
                                     const void* gate_b, const float* logits_in, int32_t E, int32_t H, int32_t I,
                                     int32_t top_k, int32_t norm_topk, const void* gu_records,
                                     const void* dn_records, int scale_dtype, int has_zeros, int32_t group,
                                     const void* residual, void* out, float* w_out, int32_t* sel_out,
                                     void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
  if (!x || !out || !gu_records || !dn_records || !workspace || (!gate_w && !logits_in)) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kGMaxT || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  if (!tc_geometry_ok(H, I, group) || g_router_smem(H) > kGSmemMax) return DUPLEX_ERR_UNSUPPORTED;
  const int N = tc_cols(T, E, top_k);
  const TcScratch L = tc_scratch(T, E, H, I, top_k, N);
  if (workspace_bytes < L.g.total) return DUPLEX_ERR_WORKSPACE;
  if (g_misaligned({x, out, workspace, gu_records, dn_records, gate_w, residual, logits_in})) return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  int* sel = reinterpret_cast<int*>(ws + L.g.sel);
  float* w = reinterpret_cast<float*>(ws + L.g.w);
  cudaStream_t st = (cudaStream_t)stream;
  const bool f16 = act_dtype == DUPLEX_DTYPE_F16;
  int rc;
  if ((rc = g_route(x, f16, T, gate_w, gate_b, logits_in, E, H, top_k, norm_topk, ws, L.g, sel, w, sel_out, w_out,
                    nullptr, 0, err, st)))
    return rc;
  return tc_expert_stage(x, (size_t)H * 2, f16, T, sel, w, top_k, top_k, 0, E, E, H, I, has_zeros, gu_records,
                         dn_records, L, N, ws, residual, out, 0, err, st, true);
}

extern "C" int duplex_moe_experts_grouped_tc_workspace_bytes(int32_t T, int32_t E_local, int32_t E_total, int32_t H,
                                                             int32_t I, int32_t top_k, int32_t group, int has_zeros,
                                                             size_t* bytes) {
  (void)has_zeros;
  if (!bytes || T < 1 || T > kGMaxT || E_local < 1 || E_total < E_local || E_total > kMaxExperts || top_k < 1 ||
      top_k > kMaxTopK || top_k > E_total)
    return DUPLEX_ERR_ARG;
  if (!tc_geometry_ok(H, I, group)) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = tc_scratch(T, E_local, H, I, top_k, tc_cols(T, E_total, top_k)).g.total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_experts_grouped_tc(const void* x, int act_dtype, int32_t T, int64_t x_row_stride,
                                             const int32_t* sel, const float* w, int32_t meta_stride, int32_t top_k,
                                             int32_t e_begin, int32_t E_local, int32_t E_total, int32_t H, int32_t I,
                                             const void* gu_records, const void* dn_records, int scale_dtype,
                                             int has_zeros, int32_t group, const void* residual, void* out,
                                             int out_dtype, void* workspace, size_t workspace_bytes, int32_t* err,
                                             void* stream) {
  if (!x || !sel || !w || !out || !gu_records || !dn_records || !workspace) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kGMaxT || E_local < 1 || e_begin < 0 || e_begin + E_local > E_total ||
      E_total > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > E_total)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (scale_dtype != act_dtype) return DUPLEX_ERR_DTYPE;
  if (out_dtype != act_dtype && out_dtype != DUPLEX_DTYPE_F32) return DUPLEX_ERR_DTYPE;
  if (!tc_geometry_ok(H, I, group)) return DUPLEX_ERR_UNSUPPORTED;
  const int N = tc_cols(T, E_total, top_k);
  const TcScratch L = tc_scratch(T, E_local, H, I, top_k, N);
  if (workspace_bytes < L.g.total) return DUPLEX_ERR_WORKSPACE;
  if (x_row_stride < H || (x_row_stride & 7)) return DUPLEX_ERR_ALIGN;
  if (meta_stride < top_k) return DUPLEX_ERR_ARG;
  if (g_misaligned({x, out, workspace, gu_records, dn_records, residual})) return DUPLEX_ERR_ALIGN;
  return tc_expert_stage(x, (size_t)x_row_stride * 2, act_dtype == DUPLEX_DTYPE_F16, T, sel, w, meta_stride, top_k,
                         e_begin, E_local, E_total, H, I, has_zeros, gu_records, dn_records, L, N,
                         reinterpret_cast<uint8_t*>(workspace), residual, out, out_dtype == DUPLEX_DTYPE_F32, err,
                         (cudaStream_t)stream, false);
}
