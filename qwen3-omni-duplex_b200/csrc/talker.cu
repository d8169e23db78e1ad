// Talker MoE (the reference's FusedMoE, src/duplex/streaming/fused_moe.py:40-141): 128
// bf16 (or per-output-channel int8) experts, top-k routing, and a shared expert whose
// output, gated by sigmoid(shared_expert_gate(x)), is added to every token:
//
//   out = sum_j round(round(y_j) * round(w_j)) + round(sigmoid(g(x)) * shared(x))
//   y_j = down_{e_j} . round(round(silu(round(gate_{e_j} . x))) * round(up_{e_j} . x))
//
// T <= 8 tokens, three launches on the caller's stream:
//   route   duplex_moe_route's kernel (moe.cu): logits rounded to the act dtype, fp32
//           softmax, top-k (ties to the lower id), renormalised when asked, and the unit
//           plan (distinct experts with their token masks);
//   gate|up one warp per (unit, intermediate row): the gate and up rows of the unit's
//           expert against every token that picked it -- each weight row is read once
//           however many tokens share the expert -- SiLU(gate) * up per (token, slot);
//           then the shared expert's rows and its gate;
//   down    one warp per output row: every selected (token, slot)'s down row against its
//           intermediate, weighted, summed over the slots in selection order, plus the
//           gated shared expert, one rounding per step as the reference's bf16 ops.
// Weights: gate_up [E][2I][H] (gate rows, then up rows), down [E][H][I], in the act dtype
// or int8 with per-row scales gu_scale [E][2I], dn_scale [E][H] (act dtype): a weight is
// round(q * s) in the act dtype, as the reference dequantises (`gu.to(dtype) * gu_s`).
// Every weight row is streamed with 16-byte loads, fp32 accumulation.
#include "common.cuh"
#include "moe.cuh"

namespace duplex {

int record_cuda(cudaError_t e);

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
    da[t] = warp_sum(da[t]);
    db[t] = warp_sum(db[t]);
  }
}

// gate|up (+ SiLU) of every (unit, row), then the shared expert's rows and its gate.
template <typename T, bool Q8, int NT>
__global__ void __launch_bounds__(kTalkThreads) talker_gateup_kernel(const __grid_constant__ TalkerParams p) {
  extern __shared__ __align__(16) float xs[];  // [T][H]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nT = NT == 1 ? 1 : p.T;
  for (int i = tid; i < nT * p.H; i += kTalkThreads)
    xs[i] = to_f32<T>(reinterpret_cast<const T*>(p.x)[i]);
  __syncthreads();
  int nU = p.plan->n_units;
  nU = nU < 0 ? 0 : (nU > kMaxUnits ? kMaxUnits : nU);
  const long long n_exp = (long long)nU * p.I;
  const long long n_items = n_exp + (p.sh_gate ? p.S : 0) + 1;
  const uint32_t all = (1u << nT) - 1u;
  for (long long it = (long long)blockIdx.x * kTalkWarps + warp; it < n_items;
       it += (long long)gridDim.x * kTalkWarps) {
    float g[NT], u[NT];
    if (it < n_exp) {
      const int un = (int)(it / p.I), i = (int)(it - (long long)un * p.I);
      int e = p.plan->unit_expert[un];
      if ((unsigned)e >= (unsigned)p.E) {  // never turn a bad id into an address
        if (lane == 0) atomicOr(p.err, DUPLEX_DEVERR_EXPERT);
        e = 0;
      }
      const uint32_t mask = p.plan->unit_mask[un] & all;
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
        const int j = slot_of(p.sel, t, p.top_k, e);
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

// down projection, weighted sum over the slots in selection order, + gated shared expert
template <typename T, bool Q8, int NT>
__global__ void __launch_bounds__(kTalkThreads) talker_down_kernel(const __grid_constant__ TalkerParams p) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nT = NT == 1 ? 1 : p.T;
  const int k = p.top_k;
  float* as = sm;                                  // [T * k][I] intermediates
  float* ss = as + (size_t)nT * k * p.I;           // [T][S] shared intermediates
  float* ps = ss + (size_t)nT * (p.sh_gate ? p.S : 0);  // [warps][T * k] weighted slot outputs
  for (int i = tid; i < nT * k * p.I; i += kTalkThreads)
    as[i] = to_f32<T>(reinterpret_cast<const T*>(p.act)[i]);
  if (p.sh_gate)
    for (int i = tid; i < nT * p.S; i += kTalkThreads)
      ss[i] = to_f32<T>(reinterpret_cast<const T*>(p.sact)[i]);
  __syncthreads();
  int nU = p.plan->n_units;
  nU = nU < 0 ? 0 : (nU > kMaxUnits ? kMaxUnits : nU);
  const uint32_t all = (1u << nT) - 1u;
  float* pw = ps + warp * kMaxTokens * kMaxTopK;
  for (int r = blockIdx.x * kTalkWarps + warp; r < p.H; r += gridDim.x * kTalkWarps) {
    for (int q = lane; q < nT * k; q += 32) pw[q] = 0.f;
    __syncwarp();
    for (int un = 0; un < nU; ++un) {
      int e = p.plan->unit_expert[un];
      if ((unsigned)e >= (unsigned)p.E) e = 0;  // reported by the gate|up kernel
      const uint32_t mask = p.plan->unit_mask[un] & all;
      const size_t row = (size_t)e * p.H + r;
      const float s = Q8 ? to_f32<T>(reinterpret_cast<const T*>(p.dn_scale)[row]) : 1.f;
      // the unit's tokens: each against its own slot's intermediate
      constexpr int N = Chunk<T, Q8>::N;
      const uint8_t* wrow = reinterpret_cast<const uint8_t*>(p.down) + row * p.I * (Q8 ? 1 : 2);
      int js[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) js[t] = ((mask >> t) & 1u) ? slot_of(p.sel, t, k, e) : -1;
      float d[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) d[t] = 0.f;
      for (int c = lane; c * N < p.I; c += 32) {
        float v[16];
        Chunk<T, Q8>::load(wrow + (size_t)c * N * (Q8 ? 1 : 2), s, v);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (js[t] < 0) continue;
          const float* ar = as + (size_t)(t * k + js[t]) * p.I + c * N;
#pragma unroll
          for (int q = 0; q < N; ++q) d[t] = fmaf(v[q], ar[q], d[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (js[t] < 0) continue;  // warp-uniform
        const float y = warp_sum(d[t]);
        if (lane == 0)
          pw[t * k + js[t]] = rnd<T>(rnd<T>(y) * rnd<T>(p.w[t * k + js[t]]));
      }
    }
    float sh[NT];
    if (p.sh_gate)
      dot2<T, false, NT>(reinterpret_cast<const uint8_t*>(p.sh_down) + (size_t)r * p.S * 2, nullptr,
                         1.f, 1.f, p.S, ss, all, lane, sh, sh);
    __syncwarp();
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (lane != t || t >= nT) continue;
      float routed = 0.f;
      for (int j = 0; j < k; ++j) routed += pw[t * k + j];
      float o = rnd<T>(routed);
      if (p.sh_gate) o += rnd<T>(p.sg[t] * rnd<T>(sh[t]));
      reinterpret_cast<T*>(p.out)[(size_t)t * p.H + r] = from_f32<T>(o);
    }
    __syncwarp();
  }
}

struct TalkerScratch {
  size_t route, act, sact, sg, w, sel, total;
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
  const int grid_a = (int)((items + kTalkWarps - 1) / kTalkWarps);
  ka<<<grid_a, kTalkThreads, smem_a, st>>>(p);
  rc = record_cuda(cudaGetLastError());
  if (rc) return rc;
  const int grid_b = (p.H + kTalkWarps - 1) / kTalkWarps;
  kb<<<grid_b, kTalkThreads, smem_b, st>>>(p);
  return record_cuda(cudaGetLastError());
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
  const size_t smem_a = (size_t)T * H * 4;
  const size_t smem_b = ((size_t)T * top_k * I + (size_t)T * (sh_gate ? S : 0)) * 4 +
                        (size_t)kTalkWarps * kMaxTokens * kMaxTopK * 4;
  if (smem_a > 227 * 1024 || smem_b > 227 * 1024) return DUPLEX_ERR_UNSUPPORTED;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* w = w_out ? w_out : reinterpret_cast<float*>(ws + L.w);
  int32_t* sel = sel_out ? sel_out : reinterpret_cast<int32_t*>(ws + L.sel);
  const MoeScratch R = moe_scratch_layout(T, E, H, 1, top_k);
  int rc = duplex_moe_route(x, act_dtype, T, gate_w, nullptr, E, H, top_k, norm_topk, w, sel,
                            ws + L.route, R.total, 0.f, 0, stream);
  if (rc) return rc;
  TalkerParams p = {};
  p.x = x; p.T = T; p.E = E; p.H = H; p.I = I; p.top_k = top_k; p.S = sh_gate ? S : 0;
  p.gate_up = gate_up; p.down = down; p.gu_scale = gu_scale; p.dn_scale = dn_scale;
  p.sh_gate = sh_gate; p.sh_up = sh_up; p.sh_down = sh_down; p.sh_gate_w = sh_gate_w;
  p.plan = reinterpret_cast<const MoePlan*>(ws + L.route + R.plan);
  p.sel = sel; p.w = w;
  p.act = ws + L.act; p.sact = ws + L.sact; p.sg = reinterpret_cast<float*>(ws + L.sg);
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
