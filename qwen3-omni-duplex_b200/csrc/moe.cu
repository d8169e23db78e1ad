// Decode MoE (T <= 8 tokens): router kernel + orchestration of the three launches.
//
// Router: one warp per expert row of the gate (E/4 CTAs of 4 warps).  The gate
// rows are loaded into registers before griddepcontrol.wait (they are weights),
// the dot products with the T token rows are done in fp32, each logit is rounded
// once into the activation dtype (nn.Linear in the module dtype,
// fused_packed_moe.py:112,195), and the CTA that arrives last on a global
// counter does, per token, softmax in fp32, top-k (ties -> lower expert id) and
// renormalisation (fused_packed_moe.py:195-199), then builds the unit plan: the
// distinct experts selected by the T tokens, each with its token mask and
// routing weights, so tokens that share an expert share one weight pass.
#include "common.cuh"
#include "moe.cuh"

#include <map>
#include <mutex>

namespace duplex {

int record_cuda(cudaError_t e);
int num_sms();
int ensure_smem_attr(const void* fn, int bytes);
int launch_moe_experts(int act_dtype, int scale_dtype, int has_zeros, int T, int E, int H, int I,
                       int group, const void* gu_tiles, const void* dn_tiles, const MoePlan* plan,
                       const void* x, void* act, const void* residual, void* out, int* err,
                       int max_units, bool pdl, cudaStream_t st);

constexpr int kRouteWarps = 4;
constexpr int kRouteMaxChunks = 16;  // 16-byte chunks per lane: H <= 16 * 32 * 8 = 4096

struct RouteParams {
  const void* x;
  const void* gate_w;
  const void* gate_b;
  int T, E, H, top_k, norm;
  float rms_eps;   // > 0: route on RMS-normalised tokens and publish them in xn
  void* xn;
  float* w_out;
  int32_t* sel_out;
  float* logits;
  int* counter;
  MoePlan* plan;
  int* err;
};

template <typename T>
DEVI void dot8(const uint4& a, const uint4& b, float& acc) {
  const T* pa = reinterpret_cast<const T*>(&a);
  const T* pb = reinterpret_cast<const T*>(&b);
#pragma unroll
  for (int q = 0; q < 8; ++q) acc = fmaf(to_f32<T>(pa[q]), to_f32<T>(pb[q]), acc);
}

template <typename T>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(const __grid_constant__ RouteParams p) {
  // dynamic smem: [gate rows of this CTA: kRouteWarps x H][tokens: T x H]
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_last;
  __shared__ int s_abort;
  __shared__ float s_ss[kRouteWarps][kMaxTokens];
  __shared__ int s_sel[kMaxTokens * kMaxTopK];
  __shared__ float s_w[kMaxTokens * kMaxTopK];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e0 = blockIdx.x * kRouteWarps;
  const int nrows = (p.E - e0) < kRouteWarps ? (p.E - e0) : kRouteWarps;
  const int nchunk = p.H >> 3;
  const uint32_t row_bytes = (uint32_t)p.H * 2u;
  uint4* wsm = reinterpret_cast<uint4*>(smem);
  uint4* xs = reinterpret_cast<uint4*>(smem + (size_t)kRouteWarps * row_bytes);

  if (tid == 0) {
    mbar_init(&bar, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // the CTA's gate rows (weights: independent of the previous kernel) in one bulk copy
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, (uint32_t)nrows * row_bytes);
    bulk_g2s(wsm, reinterpret_cast<const uint8_t*>(p.gate_w) + (size_t)e0 * row_bytes,
             (uint32_t)nrows * row_bytes, &bar);
  }
  pdl_wait();

  // token rows -> shared memory
  for (int idx = tid; idx < p.T * nchunk; idx += blockDim.x)
    xs[idx] = reinterpret_cast<const uint4*>(p.x)[idx];
  __syncthreads();
  if (p.rms_eps > 0.f) {
    // weightless RMSNorm of every token row, identical in every CTA; CTA 0 publishes
    // the normalised rows for the gate|up kernel
    T* xe = reinterpret_cast<T*>(xs);
    for (int t = 0; t < p.T; ++t) {
      float a = 0.f;
      for (int c = tid; c < p.H; c += blockDim.x) {
        const float v = to_f32<T>(xe[t * p.H + c]);
        a = fmaf(v, v, a);
      }
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) s_ss[warp][t] = a;
    }
    __syncthreads();
    for (int t = 0; t < p.T; ++t) {
      float tot = 0.f;
      for (int w = 0; w < kRouteWarps; ++w) tot += s_ss[w][t];
      const float inv = 1.0f / sqrtf(tot / (float)p.H + p.rms_eps);
      for (int c = tid; c < p.H; c += blockDim.x)
        xe[t * p.H + c] = from_f32<T>(to_f32<T>(xe[t * p.H + c]) * inv);
    }
    __syncthreads();
    if (blockIdx.x == 0 && p.xn) {
      for (int idx = tid; idx < p.T * nchunk; idx += blockDim.x)
        reinterpret_cast<uint4*>(p.xn)[idx] = xs[idx];
    }
  }
  if (!mbar_wait_bounded(&bar, 0u, &s_abort)) {
    if (tid == 0 && p.err) atomicOr(p.err, DUPLEX_DEVERR_TIMEOUT);
  }

  if (warp < nrows) {
    const int e = e0 + warp;
    float acc[kMaxTokens];
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) acc[t] = 0.f;
    const uint4* wr = wsm + (size_t)warp * nchunk;
#pragma unroll 2
    for (int c = lane; c < nchunk; c += 32) {
      const uint4 wv = wr[c];
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t)
        if (t < p.T) dot8<T>(wv, xs[t * nchunk + c], acc[t]);
    }
    for (int t = 0; t < p.T; ++t) {
      float v = acc[t];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) {
        if (p.gate_b) v += to_f32<T>(reinterpret_cast<const T*>(p.gate_b)[e]);
        p.logits[t * p.E + e] = to_f32<T>(from_f32<T>(v));
      }
    }
  }

  // ---- last CTA to arrive selects
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.counter, 1);
    s_last = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  const int per_lane = (p.E + 31) >> 5;  // <= 8
  for (int t = warp; t < p.T; t += kRouteWarps) {
    float v[8];
    unsigned taken = 0;
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ei = lane + 32 * i;
      v[i] = (i < per_lane && ei < p.E) ? __ldcg(p.logits + t * p.E + ei) : -INFINITY;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float S = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (v[i] != -INFINITY) S += expf(v[i] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);

    float pj[kMaxTopK];
    int sj[kMaxTopK];
    float psum = 0.f;
    for (int j = 0; j < p.top_k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int ei = lane + 32 * i;
        if (!((taken >> i) & 1u) && ei < p.E && (v[i] > bv || (v[i] == bv && ei < bi))) {
          bv = v[i];
          bi = ei;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      sj[j] = bi;
      pj[j] = expf(bv - m) / S;
      psum += pj[j];
    }
    if (lane == 0) {
      for (int j = 0; j < p.top_k; ++j) {
        const float w = p.norm ? pj[j] / psum : pj[j];
        p.w_out[t * p.top_k + j] = w;
        p.sel_out[t * p.top_k + j] = sj[j];
        s_w[t * kMaxTopK + j] = w;
        s_sel[t * kMaxTopK + j] = sj[j];
      }
    }
  }
  __syncthreads();

  // ---- unit plan: distinct experts in ascending id order
  if (warp == 0) {
    int base = 0;
    for (int i = 0; i < per_lane; ++i) {
      const int ei = lane + 32 * i;
      uint32_t mask = 0;
      float wv[kMaxTokens];
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t) wv[t] = 0.f;
      if (ei < p.E) {
        for (int t = 0; t < p.T; ++t)
          for (int j = 0; j < p.top_k; ++j)
            if (s_sel[t * kMaxTopK + j] == ei) {
              mask |= 1u << t;
              wv[t] = s_w[t * kMaxTopK + j];
            }
      }
      const unsigned bal = __ballot_sync(0xffffffffu, mask != 0u);
      if (mask) {
        const int pos = base + __popc(bal & ((1u << lane) - 1u));
        if (pos < kMaxUnits) {
          p.plan->unit_expert[pos] = ei;
          p.plan->unit_mask[pos] = mask;
#pragma unroll
          for (int t = 0; t < kMaxTokens; ++t) p.plan->unit_w[pos * kMaxTokens + t] = wv[t];
        }
      }
      base += __popc(bal);
    }
    if (lane == 0) {
      p.plan->n_units = base < kMaxUnits ? base : kMaxUnits;
      *p.counter = 0;  // ready for the next launch / graph replay
    }
  }
}

static inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int launch_route(int act_dtype, const RouteParams& rp, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((rp.E + kRouteWarps - 1) / kRouteWarps);
  cfg.blockDim = dim3(kRouteWarps * 32);
  cfg.dynamicSmemBytes = (size_t)(kRouteWarps + rp.T) * rp.H * 2;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (act_dtype == DUPLEX_DTYPE_F16) {
    void (*k)(RouteParams) = route_kernel<__half>;
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), 200 * 1024);
    if (rc) return rc;
    return record_cuda(cudaLaunchKernelEx(&cfg, k, rp));
  }
  if (act_dtype == DUPLEX_DTYPE_BF16) {
    void (*k)(RouteParams) = route_kernel<__nv_bfloat16>;
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), 200 * 1024);
    if (rc) return rc;
    return record_cuda(cudaLaunchKernelEx(&cfg, k, rp));
  }
  return DUPLEX_ERR_DTYPE;
}

static int check_route(const void* x, int act_dtype, int T, const void* gate_w, int E, int H,
                       int top_k, void* ws, size_t ws_bytes, int I) {
  if (I < 1) return DUPLEX_ERR_ARG;
  if (!x || !gate_w || !ws) return DUPLEX_ERR_ARG;
  if (act_dtype != DUPLEX_DTYPE_F16 && act_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E || H < 8)
    return DUPLEX_ERR_ARG;
  if ((H & 7) || H > kRouteMaxChunks * 32 * 8) return DUPLEX_ERR_UNSUPPORTED;
  if (!al16(x) || !al16(gate_w) || !al16(ws)) return DUPLEX_ERR_ALIGN;
  if (ws_bytes < moe_scratch_layout(T, E, H, I, top_k).total) return DUPLEX_ERR_WORKSPACE;
  return DUPLEX_OK;
}

static RouteParams make_route(const void* x, int T, const void* gate_w, const void* gate_b, int E,
                              int H, int top_k, int norm, float rms_eps, float* w_out,
                              int32_t* sel_out, uint8_t* ws, const MoeScratch& L) {
  RouteParams rp = {};
  rp.x = x; rp.gate_w = gate_w; rp.gate_b = gate_b;
  rp.T = T; rp.E = E; rp.H = H; rp.top_k = top_k; rp.norm = norm;
  rp.rms_eps = rms_eps;
  rp.xn = ws + L.xn;
  rp.w_out = w_out ? w_out : reinterpret_cast<float*>(ws + L.w);
  rp.sel_out = sel_out ? sel_out : reinterpret_cast<int32_t*>(ws + L.sel);
  rp.logits = reinterpret_cast<float*>(ws + L.logits);
  rp.counter = reinterpret_cast<int*>(ws + L.counter);
  rp.plan = reinterpret_cast<MoePlan*>(ws + L.plan);
  return rp;
}

// The router step of duplex_moe_forward with all of its argument checks: w / sel and
// the unit plan into the workspace.  Used by the host-resident path (staging.cu),
// which then stages the planned experts before the expert kernels run.
int moe_route_checked(const void* x, int act_dtype, int T, const void* gate_w, const void* gate_b,
                      int E, int H, int I, int top_k, int norm_topk, float* w_out,
                      int32_t* sel_out, void* workspace, size_t workspace_bytes, int* err,
                      float rms_eps, bool pdl, cudaStream_t st) {
  int rc = check_route(x, act_dtype, T, gate_w, E, H, top_k, workspace, workspace_bytes, I);
  if (rc) return rc;
  if (I < 16) return DUPLEX_ERR_ARG;
  const MoeScratch L = moe_scratch_layout(T, E, H, I, top_k);
  RouteParams rp = make_route(x, T, gate_w, gate_b, E, H, top_k, norm_topk, rms_eps, w_out,
                              sel_out, reinterpret_cast<uint8_t*>(workspace), L);
  rp.err = err;
  return launch_route(act_dtype, rp, pdl, st);
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_moe_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                          int32_t top_k, size_t* bytes) {
  if (!bytes || T < 1 || E < 1 || H < 1 || I < 1 || top_k < 1) return DUPLEX_ERR_ARG;
  *bytes = moe_scratch_layout(T, E, H, I, top_k).total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_route(const void* x, int act_dtype, int32_t T, const void* gate_w,
                                const void* gate_b, int32_t E, int32_t H, int32_t top_k,
                                int32_t norm_topk, float* w_out, int32_t* sel_out, void* workspace,
                                size_t workspace_bytes, float rms_eps, int pdl, void* stream) {
  int rc = check_route(x, act_dtype, T, gate_w, E, H, top_k, workspace, workspace_bytes, 1);
  if (rc) return rc;
  const MoeScratch L = moe_scratch_layout(T, E, H, 1, top_k);
  RouteParams rp = make_route(x, T, gate_w, gate_b, E, H, top_k, norm_topk, rms_eps, w_out,
                              sel_out, reinterpret_cast<uint8_t*>(workspace), L);
  return launch_route(act_dtype, rp, pdl != 0, (cudaStream_t)stream);
}

extern "C" int duplex_moe_forward(const void* x, int act_dtype, int32_t T, const void* gate_w,
                                  const void* gate_b, int32_t E, int32_t H, int32_t I,
                                  int32_t top_k, int32_t norm_topk, const void* gu_tiles,
                                  const void* dn_tiles, int scale_dtype, int has_zeros,
                                  int32_t group,
                                  const void* residual, void* out, float* w_out, int32_t* sel_out,
                                  void* workspace, size_t workspace_bytes, int32_t* err,
                                  float rms_eps, int pdl, void* stream) {
  int rc = check_route(x, act_dtype, T, gate_w, E, H, top_k, workspace, workspace_bytes, I);
  if (rc) return rc;
  if (!out || I < 16) return DUPLEX_ERR_ARG;
  if (!al16(out) || (residual && !al16(residual))) return DUPLEX_ERR_ALIGN;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const MoeScratch L = moe_scratch_layout(T, E, H, I, top_k);
  RouteParams rp = make_route(x, T, gate_w, gate_b, E, H, top_k, norm_topk, rms_eps, w_out,
                              sel_out, ws, L);
  rp.err = err;
  cudaStream_t st = (cudaStream_t)stream;
  rc = launch_route(act_dtype, rp, pdl != 0, st);
  if (rc) return rc;
  int max_units = T * top_k < E ? T * top_k : E;
  if (max_units > kMaxUnits) max_units = kMaxUnits;
  return launch_moe_experts(act_dtype, scale_dtype, has_zeros, T, E, H, I, group, gu_tiles,
                            dn_tiles, reinterpret_cast<const MoePlan*>(ws + L.plan),
                            rms_eps > 0.f ? (const void*)(ws + L.xn) : x, ws + L.act, residual,
                            out, err, max_units, pdl != 0, st);
}

// ---------------------------------------------------------------------------
// No-allocation variant of duplex_moe_forward.
//
// Some callers cannot call cudaMalloc (or any allocating routine) for the MoE
// scratch: a real-time frame loop such as the duplex clock path, where an
// allocation can synchronise the device and blow the 80 ms frame deadline, and
// plain C hosts that have no caching allocator to hand them a workspace.  For
// them the scratch lives in this file-scope device array instead.  It is a fixed
// kNoAllocScratchBytes per GPU, held by every GPU that loads the library until
// the process exits.  Its device address is looked up once per device with
// cudaGetSymbolAddress (on the first call made on that device, which should
// therefore happen before any stream capture).  Every call shares the array and
// finds the previous call's contents in it; the router's arrival counter is the
// only part that must start at zero and is cleared on every call.  Calls whose
// executions overlap on the GPU (different streams, or different host threads)
// race on the array and must be serialised by the caller.
namespace duplex {

constexpr size_t kNoAllocScratchBytes = (size_t)1280 * 1024;
static __device__ __align__(256) uint8_t g_moe_scratch[kNoAllocScratchBytes];

static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static std::map<int, void*> by_device;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda(e);
  std::lock_guard<std::mutex> lock(mu);
  auto it = by_device.find(dev);
  if (it == by_device.end()) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_moe_scratch);
    if (e != cudaSuccess) return record_cuda(e);
    it = by_device.emplace(dev, ptr).first;
  }
  *out = it->second;
  return DUPLEX_OK;
}

}  // namespace duplex

extern "C" size_t duplex_moe_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int duplex_moe_forward_noalloc(
    const void* x, int act_dtype, int32_t T, const void* gate_w, const void* gate_b, int32_t E,
    int32_t H, int32_t I, int32_t top_k, int32_t norm_topk, const void* gu_tiles,
    const void* dn_tiles, int scale_dtype, int has_zeros, int32_t group, const void* residual,
    void* out, float* w_out, int32_t* sel_out, int32_t* err, float rms_eps, int pdl,
    void* stream) {
  // the limits of duplex_moe_forward first, so the scratch size below cannot overflow
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E || H < 1 || I < 1)
    return DUPLEX_ERR_ARG;
  if (H > kRouteMaxChunks * 32 * 8 || I > (1 << 20)) return DUPLEX_ERR_UNSUPPORTED;
  const MoeScratch L = moe_scratch_layout(T, E, H, I, top_k);
  if (L.total > kNoAllocScratchBytes) return DUPLEX_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  // the router's arrival counter must start at zero
  rc = record_cuda(cudaMemsetAsync(reinterpret_cast<uint8_t*>(ws) + L.counter, 0, sizeof(int),
                                   (cudaStream_t)stream));
  if (rc) return rc;
  return duplex_moe_forward(x, act_dtype, T, gate_w, gate_b, E, H, I, top_k, norm_topk, gu_tiles,
                            dn_tiles, scale_dtype, has_zeros, group, residual, out, w_out,
                            sel_out, ws, kNoAllocScratchBytes, err, rms_eps, pdl, stream);
}
