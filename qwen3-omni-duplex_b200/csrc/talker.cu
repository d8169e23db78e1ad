// Talker MoE (the reference's FusedMoE, src/duplex/streaming/fused_moe.py:40-141): 128
// bf16 (or per-output-channel int8) experts, top-k routing, and a shared expert whose
// output, gated by sigmoid(shared_expert_gate(x)), is added to every token:
//
//   out = sum_j round(round(y_j) * round(w_j)) + round(sigmoid(g(x)) * shared(x))
//   y_j = down_{e_j} . round(round(silu(round(gate_{e_j} . x))) * round(up_{e_j} . x))
//
// T <= 8 tokens, four launches on the caller's stream, chained by programmatic dependent
// launch (each starts while the previous one runs and waits for it before reading its
// outputs; the shared expert's static rows are prefetched into L2 meanwhile):
//   route   duplex_moe_route's kernel (moe.cu): logits rounded to the act dtype, fp32
//           softmax, top-k (ties to the lower id), renormalised when asked, and the unit
//           plan (distinct experts with their token masks);
//   gate|up one warp per (unit, intermediate row): the gate and up rows of the unit's
//           expert against every token that picked it -- each weight row is read once
//           however many tokens share the expert -- SiLU(gate) * up per (token, slot);
//           then the shared expert's rows and its gate;
//   down    one warp per (unit, 8 output rows): the rows of the unit's expert against each
//           of its tokens' intermediates, weighted, per (token, slot); and the gated
//           shared expert per 8 output rows;
//   combine the slots summed in selection order, plus the shared expert -- one rounding
//           per step as the reference's bf16 ops.
// Weights: gate_up [E][2I][H] (gate rows, then up rows), down [E][H][I], in the act dtype
// or int8 with per-row scales gu_scale [E][2I], dn_scale [E][H] (act dtype): a weight is
// round(q * s) in the act dtype, as the reference dequantises (`gu.to(dtype) * gu_s`).
// Every weight row is streamed with 16-byte loads, fp32 accumulation.
#include "common.cuh"
#include "moe.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();

constexpr int kTalkWarps = 8;
constexpr int kTalkThreads = kTalkWarps * 32;

struct TalkerParams {
  const void* x;
  int T, E, H, I, top_k, S;
  const void* gate_up;
  const void* down;
  const void* gu_scale;   // [E][2I] (int8 weights only)
  const void* dn_scale;   // [E][H]
  const void* sh_gate;    // [S][H] shared expert, or null
  const void* sh_up;      // [S][H]
  const void* sh_down;    // [H][S]
  const void* sh_gate_w;  // [H] shared_expert_gate, or null (gate 1)
  const MoePlan* plan;
  const int32_t* sel;     // [T][top_k]
  const float* w;         // [T][top_k]
  void* act;              // [T * top_k][I] act dtype
  void* sact;             // [T][S] act dtype
  float* sg;              // [T] the shared gate, rounded to the act dtype
  float* ypart;           // [T * top_k][H] each (token, slot)'s weighted down output
  float* shpart;          // [T][H] the gated shared expert's output
  void* out;              // [T][H]
  int* err;
};

template <typename T>
DEVI float rnd(float v) { return to_f32<T>(from_f32<T>(v)); }

template <typename T>
DEVI float silu_r(float g) {  // round(silu(g)) in T, as F.silu on a T tensor
  return rnd<T>(g / (1.0f + expf(-g)));
}

// 16 bytes of one weight row as floats: 8 values of T, or 16 int8 values dequantised
// to round(q * s) in T.
template <typename T, bool Q8>
struct Chunk {
  static constexpr int N = Q8 ? 16 : 8;
  DEVI static void load(const uint8_t* p, float s, float (&v)[16]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    if (Q8) {
      const int8_t* q = reinterpret_cast<const int8_t*>(&u);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = rnd<T>((float)q[k] * s);
    } else {
      const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = to_f32<T>(h[k]);
    }
  }
};

// L2 prefetch of `bytes` (a multiple of 16) at a 16-byte aligned global address (no
// shared memory written, nothing waits on it).
DEVI void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

DEVI float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// slot of expert e in token t's selection (-1 if absent)
DEVI int slot_of(const int32_t* sel, int t, int k, int e) {
  for (int j = 0; j < k; ++j)
    if (sel[t * k + j] == e) return j;
  return -1;
}

// The plan in shared memory: the units' experts (ue) and token masks (um), and
// jt[u * kMaxTokens + t] = the slot of unit u's expert in token t's selection (-1 when t
// did not pick it).  The selection and the plan are read from global memory once, with
// one load per thread; the table is built from shared memory.  `scr` holds the
// selection (kMaxTokens * kMaxTopK ints).  Starts and ends with a CTA barrier.
DEVI void plan_table(const MoePlan* plan, int nU, const int32_t* sel, int nT, int k, int* ue,
                     uint32_t* um, int* jt, int* scr) {
  for (int q = threadIdx.x; q < kMaxUnits; q += blockDim.x) {
    ue[q] = q < nU ? plan->unit_expert[q] : -1;
    um[q] = q < nU ? plan->unit_mask[q] : 0u;
  }
  for (int q = threadIdx.x; q < nT * k; q += blockDim.x) scr[q] = sel[q];
  __syncthreads();
  for (int q = threadIdx.x; q < kMaxUnits * kMaxTokens; q += blockDim.x) {
    const int u = q / kMaxTokens, t = q - u * kMaxTokens;
    int j = -1;
    if (u < nU && t < nT && ((um[u] >> t) & 1u)) j = slot_of(scr, t, k, ue[u]);
    jt[q] = j;
  }
  __syncthreads();
}

// shared-memory bytes of plan_table's arrays (ue, um, jt, scr)
constexpr int kPlanTableBytes = 4 * (2 * kMaxUnits + kMaxUnits * kMaxTokens + kMaxTokens * kMaxTopK);

// dots of rows a and b (K values, 16-byte chunks) with the tokens of `mask`; xs [NT][K]
// floats in shared memory.  Lanes take chunks lane, lane + 32, ...
template <typename T, bool Q8, int NT>
DEVI void dot2(const uint8_t* a, const uint8_t* b, float sa, float sb, int K, const float* xs,
               uint32_t mask, int lane, float (&da)[NT], float (&db)[NT]) {
  constexpr int N = Chunk<T, Q8>::N;
  const int ebytes = Q8 ? 1 : 2;
#pragma unroll
  for (int t = 0; t < NT; ++t) da[t] = db[t] = 0.f;
  for (int c = lane; c * N < K; c += 32) {
    float va[16], vb[16];
    Chunk<T, Q8>::load(a + (size_t)c * N * ebytes, sa, va);
    if (b) Chunk<T, Q8>::load(b + (size_t)c * N * ebytes, sb, vb);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (!((mask >> t) & 1u)) continue;
      const float* xr = xs + (size_t)t * K + c * N;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        da[t] = fmaf(va[k], xr[k], da[t]);
        if (b) db[t] = fmaf(vb[k], xr[k], db[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    if (!((mask >> t) & 1u)) continue;  // warp-uniform
    da[t] = warp_sum(da[t]);
    if (b) db[t] = warp_sum(db[t]);
  }
}

// gate|up (+ SiLU) of every (unit, row), then the shared expert's rows and its gate.
template <typename T, bool Q8, int NT>
__global__ void __launch_bounds__(kTalkThreads) talker_gateup_kernel(const __grid_constant__ TalkerParams p) {
  extern __shared__ __align__(16) float xs[];  // [T][H], then the slot table
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nT = NT == 1 ? 1 : p.T;
  pdl_launch_dependents();
  // the shared expert's rows are static: pull this CTA's share into L2 while the router
  // runs (launched with programmatic dependent launch)
  if (p.sh_gate && tid < 2) {
    const int per = (p.S + gridDim.x - 1) / gridDim.x, r0 = blockIdx.x * per;
    const int nr = r0 >= p.S ? 0 : (p.S - r0 < per ? p.S - r0 : per);
    if (nr > 0)
      prefetch_l2(reinterpret_cast<const uint8_t*>(tid ? p.sh_up : p.sh_gate) + (size_t)r0 * p.H * 2,
                  (uint32_t)nr * p.H * 2);
  }
  pdl_wait();
  int nU = p.plan->n_units;
  nU = nU < 0 ? 0 : (nU > kMaxUnits ? kMaxUnits : nU);
  int* ue = reinterpret_cast<int*>(xs + (size_t)nT * p.H);
  uint32_t* um = reinterpret_cast<uint32_t*>(ue + kMaxUnits);
  int* jt = reinterpret_cast<int*>(um + kMaxUnits);
  {
    const uint4* src = reinterpret_cast<const uint4*>(p.x);
    for (int i = tid; i < (nT * p.H) / 8; i += kTalkThreads) {
      const uint4 v = src[i];
      const T* h8 = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int z = 0; z < 8; ++z) xs[i * 8 + z] = to_f32<T>(h8[z]);
    }
  }
  plan_table(p.plan, nU, p.sel, nT, p.top_k, ue, um, jt, jt + kMaxUnits * kMaxTokens);
  const long long n_exp = (long long)nU * p.I;
  const long long n_items = n_exp + (p.sh_gate ? p.S : 0) + 1;
  const uint32_t all = (1u << nT) - 1u;
  for (long long it = (long long)blockIdx.x * kTalkWarps + warp; it < n_items;
       it += (long long)gridDim.x * kTalkWarps) {
    float g[NT], u[NT];
    if (it < n_exp) {
      const int un = (int)(it / p.I), i = (int)(it - (long long)un * p.I);
      int e = ue[un];
      if ((unsigned)e >= (unsigned)p.E) {  // never turn a bad id into an address
        if (lane == 0) atomicOr(p.err, DUPLEX_DEVERR_EXPERT);
        e = 0;
      }
      const uint32_t mask = um[un] & all;
      const size_t eb = Q8 ? 1 : 2;
      const uint8_t* base = reinterpret_cast<const uint8_t*>(p.gate_up);
      const size_t rg = (size_t)e * 2 * p.I + i, ru = rg + p.I;
      float sa = 1.f, sb = 1.f;
      if (Q8) {
        sa = to_f32<T>(reinterpret_cast<const T*>(p.gu_scale)[rg]);
        sb = to_f32<T>(reinterpret_cast<const T*>(p.gu_scale)[ru]);
      }
      dot2<T, Q8, NT>(base + rg * p.H * eb, base + ru * p.H * eb, sa, sb, p.H, xs, mask, lane, g, u);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (lane != t || !((mask >> t) & 1u)) continue;
        const int j = jt[un * kMaxTokens + t];
        if (j < 0) continue;
        const float a = rnd<T>(silu_r<T>(rnd<T>(g[t])) * rnd<T>(u[t]));
        reinterpret_cast<T*>(p.act)[(size_t)(t * p.top_k + j) * p.I + i] = from_f32<T>(a);
      }
    } else if (it < n_items - 1) {
      const int i = (int)(it - n_exp);
      dot2<T, false, NT>(reinterpret_cast<const uint8_t*>(p.sh_gate) + (size_t)i * p.H * 2,
                         reinterpret_cast<const uint8_t*>(p.sh_up) + (size_t)i * p.H * 2, 1.f, 1.f,
                         p.H, xs, all, lane, g, u);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (lane == t && t < nT) {
          const float a = rnd<T>(silu_r<T>(rnd<T>(g[t])) * rnd<T>(u[t]));
          reinterpret_cast<T*>(p.sact)[(size_t)t * p.S + i] = from_f32<T>(a);
        }
    } else {
      // the shared expert's gate: sigmoid(round(x . g)) rounded, per token (1 without one)
      if (p.sh_gate_w)
        dot2<T, false, NT>(reinterpret_cast<const uint8_t*>(p.sh_gate_w), nullptr, 1.f, 1.f, p.H,
                           xs, all, lane, g, u);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (lane == t && t < nT)
          p.sg[t] = p.sh_gate_w ? rnd<T>(1.0f / (1.0f + expf(-rnd<T>(g[t])))) : 1.f;
    }
  }
}

// down projection, weighted sum over the slots in selection order, + gated shared expert.
// A CTA takes kTalkRows output rows; its warps share the (unit, row) dot products, two
// at a time so that two rows' loads are in flight per lane, and put each selected
// (token, slot)'s weighted output round(round(y) * round(w)) into shared memory; warp w
// then takes row w's shared expert, and a last pass sums the slots in selection order.
// output rows of one down item: 8 for one token, 4 for up to 8 (registers: 2 CTAs per SM)
template <int NT>
struct Blk { static constexpr int kRows = NT == 1 ? 8 : 4; };

// values [8 h, 8 h + 8) of a 16-byte weight chunk as floats: int8 dequantised to
// round(q * s) in T (h = 0, 1), or the 8 values of T (h = 0)
template <typename T, bool Q8>
DEVI void deq8(const uint4& raw, int h, float s, float (&w)[8]) {
  if (Q8) {
    const int8_t* q = reinterpret_cast<const int8_t*>(&raw) + 8 * h;
#pragma unroll
    for (int z = 0; z < 8; ++z) w[z] = rnd<T>((float)q[z] * s);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int z = 0; z < 8; ++z) w[z] = to_f32<T>(e[z]);
  }
}

// 8 values of T at a 16-byte aligned global address (read-only path) as floats
template <typename T>
DEVI void ld8(const void* src, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int z = 0; z < 8; ++z) v[z] = to_f32<T>(h[z]);
}

// down projection.  An item is (unit, block of kTalkBlk output rows) -- kTalkBlk
// consecutive rows of the unit's expert, one contiguous stretch of weights, all in
// flight at once, each intermediate chunk reused for every row -- or (shared expert,
// row block).  Every selected (token, slot) gets round(round(y) * round(w)) in ypart;
// the shared expert round(gate * round(y)) in shpart.  Persistent CTAs walk the items.
template <typename T, bool Q8, int NT>
__global__ void __launch_bounds__(kTalkThreads, 2) talker_down_kernel(const __grid_constant__ TalkerParams p) {
  constexpr int kTalkBlk = Blk<NT>::kRows;
  extern __shared__ __align__(16) uint8_t smb[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nT = NT == 1 ? 1 : p.T;
  const int k = p.top_k;
  const int S = p.sh_gate ? p.S : 0;
  const int nblk = (p.H + kTalkBlk - 1) / kTalkBlk;
  pdl_launch_dependents();
  if (S && tid == 0) {  // the shared expert's static rows into L2 while the gate|up kernel runs
    const int per = (nblk + gridDim.x - 1) / gridDim.x, b0 = blockIdx.x * per;
    const int rb = b0 * kTalkBlk, re = (b0 + per) * kTalkBlk < p.H ? (b0 + per) * kTalkBlk : p.H;
    if (rb < re)
      prefetch_l2(reinterpret_cast<const uint8_t*>(p.sh_down) + (size_t)rb * S * 2,
                  (uint32_t)(re - rb) * S * 2);
  }
  pdl_wait();
  int* ue = reinterpret_cast<int*>(smb);
  uint32_t* um = reinterpret_cast<uint32_t*>(ue + kMaxUnits);
  int* jt = reinterpret_cast<int*>(um + kMaxUnits);
  int nU = p.plan->n_units;
  nU = nU < 0 ? 0 : (nU > kMaxUnits ? kMaxUnits : nU);
  plan_table(p.plan, nU, p.sel, nT, k, ue, um, jt, jt + kMaxUnits * kMaxTokens);
  const T* act = reinterpret_cast<const T*>(p.act);
  const uint32_t all = (1u << nT) - 1u;
  constexpr int N = Chunk<T, Q8>::N;
  const int eb = Q8 ? 1 : 2;
  const int n_unit_items = nU * nblk;
  const int n_items = n_unit_items + (S ? nblk : 0);
  for (int it = blockIdx.x * kTalkWarps + warp; it < n_items; it += gridDim.x * kTalkWarps) {
    float acc[kTalkBlk][NT];
#pragma unroll
    for (int r = 0; r < kTalkBlk; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    if (it < n_unit_items) {
      const int un = it / nblk, r0 = (it - un * nblk) * kTalkBlk;
      int e = ue[un];
      if ((unsigned)e >= (unsigned)p.E) e = 0;  // reported by the gate|up kernel
      const uint32_t mask = um[un] & all;
      int js[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) js[t] = ((mask >> t) & 1u) ? jt[un * kMaxTokens + t] : -1;
      const uint8_t* w0 = reinterpret_cast<const uint8_t*>(p.down) + ((size_t)e * p.H + r0) * p.I * eb;
      float sc[kTalkBlk];
#pragma unroll
      for (int r = 0; r < kTalkBlk; ++r)
        sc[r] = (Q8 && r0 + r < p.H)
                    ? to_f32<T>(reinterpret_cast<const T*>(p.dn_scale)[(size_t)e * p.H + r0 + r]) : 1.f;
      for (int c = lane; c * N < p.I; c += 32) {
        uint4 raw[kTalkBlk];  // the rows. chunks, all loads in flight before any use
#pragma unroll
        for (int r = 0; r < kTalkBlk; ++r)
          raw[r] = r0 + r < p.H
                       ? __ldg(reinterpret_cast<const uint4*>(w0 + ((size_t)r * p.I + (size_t)c * N) * eb))
                       : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (js[t] < 0) continue;
          const T* ar = act + (size_t)(t * k + js[t]) * p.I + c * N;
#pragma unroll
          for (int m = 0; m < N; m += 8) {
            float a8[8];
            ld8<T>(ar + m, a8);
#pragma unroll
            for (int r = 0; r < kTalkBlk; ++r) {
              float w8[8];
              deq8<T, Q8>(raw[r], m >> 3, sc[r], w8);
#pragma unroll
              for (int z = 0; z < 8; ++z) acc[r][t] = fmaf(w8[z], a8[z], acc[r][t]);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (js[t] < 0) continue;  // warp-uniform
        const float wr = rnd<T>(p.w[t * k + js[t]]);
#pragma unroll
        for (int r = 0; r < kTalkBlk; ++r) {
          const float y = warp_sum(acc[r][t]);
          if (lane == r && r0 + r < p.H)
            p.ypart[(size_t)(t * k + js[t]) * p.H + r0 + r] = rnd<T>(rnd<T>(y) * wr);
        }
      }
    } else {
      const int r0 = (it - n_unit_items) * kTalkBlk;
      const uint8_t* w0 = reinterpret_cast<const uint8_t*>(p.sh_down) + (size_t)r0 * S * 2;
      const T* sa = reinterpret_cast<const T*>(p.sact);
      for (int c = lane; c * 8 < S; c += 32) {
        uint4 raw[kTalkBlk];
#pragma unroll
        for (int r = 0; r < kTalkBlk; ++r)
          raw[r] = r0 + r < p.H
                       ? __ldg(reinterpret_cast<const uint4*>(w0 + ((size_t)r * S + (size_t)c * 8) * 2))
                       : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= nT) continue;
          float a8[8];
          ld8<T>(sa + (size_t)t * S + c * 8, a8);
#pragma unroll
          for (int r = 0; r < kTalkBlk; ++r) {
            float w8[8];
            deq8<T, false>(raw[r], 0, 1.f, w8);
#pragma unroll
            for (int z = 0; z < 8; ++z) acc[r][t] = fmaf(w8[z], a8[z], acc[r][t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= nT) continue;
#pragma unroll
        for (int r = 0; r < kTalkBlk; ++r) {
          const float y = warp_sum(acc[r][t]);
          if (lane == r && r0 + r < p.H) p.shpart[(size_t)t * p.H + r0 + r] = rnd<T>(p.sg[t] * rnd<T>(y));
        }
      }
    }
  }
}

// out[t][r] = round(round(sum_j ypart[t * k + j][r]) + shpart[t][r]): the slots in
// selection order.
template <typename T>
__global__ void __launch_bounds__(kTalkThreads) talker_combine_kernel(const __grid_constant__ TalkerParams p) {
  pdl_wait();
  const int nT = p.T, k = p.top_k;
  for (int i = blockIdx.x * kTalkThreads + threadIdx.x; i < nT * p.H; i += gridDim.x * kTalkThreads) {
    const int t = i / p.H, r = i - t * p.H;
    float routed = 0.f;
    for (int j = 0; j < k; ++j) routed += p.ypart[(size_t)(t * k + j) * p.H + r];
    float o = rnd<T>(routed);
    if (p.sh_gate) o += p.shpart[i];
    reinterpret_cast<T*>(p.out)[i] = from_f32<T>(o);
  }
}

struct TalkerScratch {
  size_t route, act, sact, sg, w, sel, ypart, shpart, total;
};

static TalkerScratch talker_scratch(int T, int E, int H, int I, int top_k, int S) {
  TalkerScratch s;
  const MoeScratch r = moe_scratch_layout(T, E, H, 1, top_k);
  size_t off = 0;
  s.route = off; off += align_up(r.total, 256);
  s.act = off; off += align_up((size_t)T * top_k * I * 2, 256);
  s.sact = off; off += align_up((size_t)T * (S > 0 ? S : 1) * 2, 256);
  s.sg = off; off += 256;
  s.w = off; off += align_up((size_t)T * top_k * 4, 256);
  s.sel = off; off += align_up((size_t)T * top_k * 4, 256);
  s.ypart = off; off += align_up((size_t)T * top_k * H * 4, 256);
  s.shpart = off; off += align_up((size_t)T * H * 4, 256);
  s.total = off;
  return s;
}

template <typename T, bool Q8, int NT>
static int launch_talker(const TalkerParams& p, size_t smem_a, size_t smem_b, cudaStream_t st) {
  auto ka = talker_gateup_kernel<T, Q8, NT>;
  auto kb = talker_down_kernel<T, Q8, NT>;
  int rc = record_cuda(cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_a));
  if (rc) return rc;
  rc = record_cuda(cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b));
  if (rc) return rc;
  int max_units = p.T * p.top_k < p.E ? p.T * p.top_k : p.E;
  if (max_units > kMaxUnits) max_units = kMaxUnits;
  const long long items = (long long)max_units * p.I + (p.sh_gate ? p.S : 0) + 1;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kTalkThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent grids: as many CTAs as can be resident walk the items (the per-CTA set-up
  // -- the tokens, the plan table -- is paid once per CTA, in one wave)
  int occ_a = 0, occ_b = 0;
  rc = record_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_a, ka, kTalkThreads, smem_a));
  if (rc) return rc;
  rc = record_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_b, kb, kTalkThreads, smem_b));
  if (rc) return rc;
  const long long cap_a = (long long)num_sms() * (occ_a > 0 ? occ_a : 1);
  const long long cap_b = (long long)num_sms() * (occ_b > 0 ? occ_b : 1);
  long long ga = (items + kTalkWarps - 1) / kTalkWarps;
  cfg.gridDim = dim3((unsigned)(ga < cap_a ? ga : cap_a));
  cfg.dynamicSmemBytes = smem_a;
  rc = record_cuda(cudaLaunchKernelEx(&cfg, ka, p));
  if (rc) return rc;
  const long long nblk = (p.H + Blk<NT>::kRows - 1) / Blk<NT>::kRows;
  long long gb = ((long long)max_units * nblk + (p.sh_gate ? nblk : 0) + kTalkWarps - 1) / kTalkWarps;
  cfg.gridDim = dim3((unsigned)(gb < cap_b ? gb : cap_b));
  cfg.dynamicSmemBytes = smem_b;
  rc = record_cuda(cudaLaunchKernelEx(&cfg, kb, p));
  if (rc) return rc;
  cfg.gridDim = dim3((unsigned)((p.T * p.H + kTalkThreads - 1) / kTalkThreads));
  cfg.dynamicSmemBytes = 0;
  return record_cuda(cudaLaunchKernelEx(&cfg, talker_combine_kernel<T>, p));
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_talker_moe_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                                 int32_t top_k, int32_t S, size_t* bytes) {
  if (!bytes || T < 1 || E < 1 || H < 1 || I < 1 || top_k < 1 || S < 0) return DUPLEX_ERR_ARG;
  *bytes = talker_scratch(T, E, H, I, top_k, S).total;
  return DUPLEX_OK;
}

extern "C" int duplex_talker_moe_forward(
    const void* x, int act_dtype, int32_t T, const void* gate_w, int32_t E, int32_t H,
    int32_t I, int32_t top_k, int32_t norm_topk, const void* gate_up, const void* down,
    int weight_int8, const void* gu_scale, const void* dn_scale, const void* sh_gate,
    const void* sh_up, const void* sh_down, int32_t S, const void* sh_gate_w, void* out,
    float* w_out, int32_t* sel_out, void* workspace, size_t workspace_bytes, int32_t* err,
    void* stream) {
  if (!x || !gate_w || !gate_up || !down || !out || !workspace || !err) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E || H < 8 || I < 8 || S < 0)
    return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (weight_int8 && (!gu_scale || !dn_scale)) return DUPLEX_ERR_ARG;
  if (sh_gate && (!sh_up || !sh_down || S < 8)) return DUPLEX_ERR_ARG;
  // 16-byte rows: H, I (and S) multiples of 8 (act-dtype rows) or 16 (int8 rows)
  const int mult = weight_int8 ? 16 : 8;
  if (H % mult || I % mult || H % 8 || (sh_gate && S % 8)) return DUPLEX_ERR_ALIGN;
  const void* ptrs[] = {x, gate_up, down, sh_gate, sh_up, sh_down, sh_gate_w, out, workspace};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return DUPLEX_ERR_ALIGN;
  const TalkerScratch L = talker_scratch(T, E, H, I, top_k, sh_gate ? S : 0);
  if (workspace_bytes < L.total) return DUPLEX_ERR_WORKSPACE;
  const size_t smem_a = (size_t)T * H * 4 + kPlanTableBytes;
  const size_t smem_b = kPlanTableBytes;
  if (smem_a > 227 * 1024 || smem_b > 227 * 1024) return DUPLEX_ERR_UNSUPPORTED;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* w = w_out ? w_out : reinterpret_cast<float*>(ws + L.w);
  int32_t* sel = sel_out ? sel_out : reinterpret_cast<int32_t*>(ws + L.sel);
  const MoeScratch R = moe_scratch_layout(T, E, H, 1, top_k);
  int rc = duplex_moe_route(x, act_dtype, T, gate_w, nullptr, E, H, top_k, norm_topk, w, sel,
                            ws + L.route, R.total, 0.f, 1, stream);
  if (rc) return rc;
  TalkerParams p = {};
  p.x = x; p.T = T; p.E = E; p.H = H; p.I = I; p.top_k = top_k; p.S = sh_gate ? S : 0;
  p.gate_up = gate_up; p.down = down; p.gu_scale = gu_scale; p.dn_scale = dn_scale;
  p.sh_gate = sh_gate; p.sh_up = sh_up; p.sh_down = sh_down; p.sh_gate_w = sh_gate_w;
  p.plan = reinterpret_cast<const MoePlan*>(ws + L.route + R.plan);
  p.sel = sel; p.w = w;
  p.act = ws + L.act; p.sact = ws + L.sact; p.sg = reinterpret_cast<float*>(ws + L.sg);
  p.ypart = reinterpret_cast<float*>(ws + L.ypart);
  p.shpart = reinterpret_cast<float*>(ws + L.shpart);
  p.out = out; p.err = err;
  cudaStream_t st = (cudaStream_t)stream;
  const bool one = T == 1;
  if (act_dtype == DUPLEX_DTYPE_F16) {
    using H16 = __half;
    if (weight_int8)
      return one ? launch_talker<H16, true, 1>(p, smem_a, smem_b, st)
                 : launch_talker<H16, true, kMaxTokens>(p, smem_a, smem_b, st);
    return one ? launch_talker<H16, false, 1>(p, smem_a, smem_b, st)
               : launch_talker<H16, false, kMaxTokens>(p, smem_a, smem_b, st);
  }
  using B16 = __nv_bfloat16;
  if (weight_int8)
    return one ? launch_talker<B16, true, 1>(p, smem_a, smem_b, st)
               : launch_talker<B16, true, kMaxTokens>(p, smem_a, smem_b, st);
  return one ? launch_talker<B16, false, 1>(p, smem_a, smem_b, st)
             : launch_talker<B16, false, kMaxTokens>(p, smem_a, smem_b, st);
}
