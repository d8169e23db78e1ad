// Host-resident experts: the reference's `host_resident=True` layers
// (src/duplex/streaming/fused_packed_moe.py:130-164 and :233-253).
//
// The reference keeps each expert's packed tensors in pinned host RAM as two byte
// blobs (gate|up, down).  For every token it reads the selection back to the host
// (`sel.tolist()`, a device synchronisation), issues one host-to-device copy per
// selected expert and blob into a k-slot staging buffer, and runs its GEMVs on the
// staged slots with the selection replaced by 0..k-1.
//
// Here the experts' tile records (the kernels' own layout, built once on the GPU)
// live in MAPPED pinned host memory (cudaHostAllocMapped: the GPU reads it over the
// host link with ordinary loads), and one call runs, all on the caller's stream:
//   1. the router kernel of duplex_moe_forward: w / sel and the unit plan (the
//      distinct experts of the <= 8 tokens);
//   2. stage_kernel: for every planned unit u, its expert's gate|up and down records
//      are read from host memory with 16-byte loads (several in flight per thread)
//      and written into device slot u; a copy of the plan names slot u as the
//      unit's expert;
//   3. the gate|up and down kernels of duplex_moe_forward on the slots.
// There is no host synchronisation and no per-expert launch, so a staged layer can
// be captured in a CUDA graph like a resident one.  The expert kernels read the same
// record bytes as on the resident path, so the output is bit-identical to
// duplex_moe_forward on device-resident records.
#include "common.cuh"
#include "moe.cuh"
#include "tiles.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int moe_route_checked(const void* x, int act_dtype, int T, const void* gate_w, const void* gate_b,
                      int E, int H, int I, int top_k, int norm_topk, float* w_out,
                      int32_t* sel_out, void* workspace, size_t workspace_bytes, int* err,
                      float rms_eps, bool pdl, cudaStream_t st);
int launch_moe_experts(int act_dtype, int scale_dtype, int has_zeros, int T, int E, int H, int I,
                       int group, const void* gu_tiles, const void* dn_tiles, const MoePlan* plan,
                       const void* x, void* act, const void* residual, void* out, int* err,
                       int max_units, bool pdl, cudaStream_t st);

constexpr int kStageThreads = 256;
constexpr int kStageCtasPerUnit = 32;  // 8 units x 32 CTAs at one token: ~256 CTAs of loads

// The staging buffer: [staged plan][gate|up slots][down slots], 256-byte aligned parts.
struct StageLayout {
  size_t gu_expert, dn_expert;  // record bytes of one expert (gate|up, down)
  size_t plan, gu, dn, total;
};

static bool stage_layout(int H, int I, int group, int has_zeros, int slots, StageLayout* s) {
  TileGeom gg, dg;
  if (tile_geom(H, group, has_zeros, &gg) || tile_geom(I, group, has_zeros, &dg)) return false;
  s->gu_expert = (size_t)(2 * I / 16) * gg.rec_bytes;
  s->dn_expert = (size_t)((H + 15) / 16) * dg.rec_bytes;
  size_t off = 0;
  s->plan = off;
  off += align_up(sizeof(MoePlan), 256);
  s->gu = off;
  off += align_up(s->gu_expert * (size_t)slots, 256);
  s->dn = off;
  off += align_up(s->dn_expert * (size_t)slots, 256);
  s->total = off;
  return true;
}

static int stage_slots(int T, int E, int top_k) {
  int s = T * top_k < E ? T * top_k : E;
  return s < kMaxUnits ? s : kMaxUnits;
}

// n16 16-byte pieces from src to dst, this thread taking pieces first, first + step, ...,
// four loads in flight before their stores (host-link latency is several microseconds)
DEVI void copy_pieces(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n16,
                      size_t first, size_t step) {
  size_t q = first;
  for (; q + 3 * step < n16; q += 4 * step) {
    const uint4 a = src[q], b = src[q + step], c = src[q + 2 * step], d = src[q + 3 * step];
    dst[q] = a;
    dst[q + step] = b;
    dst[q + 2 * step] = c;
    dst[q + 3 * step] = d;
  }
  for (; q < n16; q += step) dst[q] = src[q];
}

// Grid (slots, kStageCtasPerUnit).  CTA (u, c) copies its share of unit u's records;
// CTA (u, 0) also writes unit u of the staged plan, CTA (0, 0) the unit count.  Units
// past the plan's count exit at once.  An expert id outside [0, E) (which the router
// never writes) sets DUPLEX_DEVERR_EXPERT and stages nothing for that unit.
__global__ void __launch_bounds__(kStageThreads) stage_kernel(
    const MoePlan* __restrict__ plan, MoePlan* __restrict__ staged, const uint8_t* gu_host,
    const uint8_t* dn_host, size_t gu_expert, size_t dn_expert, int E,
    uint8_t* __restrict__ gu_slots, uint8_t* __restrict__ dn_slots, int* err) {
  const int u = blockIdx.x;
  int n = plan->n_units;  // <= slots (= gridDim.x) by construction; clamped all the same
  n = n < 0 ? 0 : (n > (int)gridDim.x ? (int)gridDim.x : n);
  if (u == 0 && blockIdx.y == 0 && threadIdx.x == 0) staged->n_units = n;
  if (u >= n) return;
  const int e = plan->unit_expert[u];
  if (blockIdx.y == 0) {
    if (threadIdx.x < kMaxTokens)
      staged->unit_w[u * kMaxTokens + threadIdx.x] = plan->unit_w[u * kMaxTokens + threadIdx.x];
    if (threadIdx.x == 0) {
      staged->unit_expert[u] = u;
      staged->unit_mask[u] = plan->unit_mask[u];
      if ((unsigned)e >= (unsigned)E && err) set_error(err, DUPLEX_DEVERR_EXPERT);
    }
  }
  if ((unsigned)e >= (unsigned)E) return;
  const size_t first = (size_t)blockIdx.y * blockDim.x + threadIdx.x;
  const size_t step = (size_t)gridDim.y * blockDim.x;
  copy_pieces(reinterpret_cast<const uint4*>(gu_host + (size_t)e * gu_expert),
              reinterpret_cast<uint4*>(gu_slots + (size_t)u * gu_expert), gu_expert >> 4, first,
              step);
  copy_pieces(reinterpret_cast<const uint4*>(dn_host + (size_t)e * dn_expert),
              reinterpret_cast<uint4*>(dn_slots + (size_t)u * dn_expert), dn_expert >> 4, first,
              step);
}

static inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_host_alloc(size_t bytes, void** host_ptr, void** dev_ptr) {
  if (!host_ptr || !dev_ptr || bytes == 0) return DUPLEX_ERR_ARG;
  void* h = nullptr;
  int rc = record_cuda(cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
  if (rc) return rc;
  void* d = nullptr;
  rc = record_cuda(cudaHostGetDevicePointer(&d, h, 0));
  if (rc) {
    cudaFreeHost(h);
    return rc;
  }
  *host_ptr = h;
  *dev_ptr = d;
  return DUPLEX_OK;
}

extern "C" int duplex_host_free(void* host_ptr) {
  if (!host_ptr) return DUPLEX_ERR_ARG;
  return record_cuda(cudaFreeHost(host_ptr));
}

extern "C" int duplex_moe_stage_bytes(int32_t T, int32_t E, int32_t H, int32_t I, int32_t top_k,
                                      int32_t group, int has_zeros, size_t* bytes) {
  if (!bytes || T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 ||
      top_k > kMaxTopK || top_k > E || H < 1 || I < 16)
    return DUPLEX_ERR_ARG;
  StageLayout S;
  if (!stage_layout(H, I, group, has_zeros, stage_slots(T, E, top_k), &S))
    return DUPLEX_ERR_UNSUPPORTED;
  *bytes = S.total;
  return DUPLEX_OK;
}

extern "C" int duplex_moe_forward_staged(
    const void* x, int act_dtype, int32_t T, const void* gate_w, const void* gate_b, int32_t E,
    int32_t H, int32_t I, int32_t top_k, int32_t norm_topk, const void* gu_tiles_host,
    const void* dn_tiles_host, int scale_dtype, int has_zeros, int32_t group,
    const void* residual, void* out, float* w_out, int32_t* sel_out, void* workspace,
    size_t workspace_bytes, void* stage, size_t stage_bytes, int32_t* err, float rms_eps,
    int pdl, void* stream) {
  if (!out || !gu_tiles_host || !dn_tiles_host || !stage) return DUPLEX_ERR_ARG;
  if (T < 1 || T > kMaxTokens || E < 1 || E > kMaxExperts || top_k < 1 || top_k > kMaxTopK ||
      top_k > E || H < 1 || I < 16)
    return DUPLEX_ERR_ARG;
  if (!al16(out) || (residual && !al16(residual)) || !al16(stage) || !al16(gu_tiles_host) ||
      !al16(dn_tiles_host))
    return DUPLEX_ERR_ALIGN;
  const int slots = stage_slots(T, E, top_k);
  StageLayout S;
  if (!stage_layout(H, I, group, has_zeros, slots, &S)) return DUPLEX_ERR_UNSUPPORTED;
  if (stage_bytes < S.total) return DUPLEX_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = moe_route_checked(x, act_dtype, T, gate_w, gate_b, E, H, I, top_k, norm_topk, w_out,
                             sel_out, workspace, workspace_bytes, err, rms_eps, pdl != 0, st);
  if (rc) return rc;
  const MoeScratch L = moe_scratch_layout(T, E, H, I, top_k);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  uint8_t* sb = reinterpret_cast<uint8_t*>(stage);
  MoePlan* staged = reinterpret_cast<MoePlan*>(sb + S.plan);
  // plain stream order after the router (no programmatic launch): the copies need its plan
  stage_kernel<<<dim3((unsigned)slots, kStageCtasPerUnit), kStageThreads, 0, st>>>(
      reinterpret_cast<const MoePlan*>(ws + L.plan), staged,
      reinterpret_cast<const uint8_t*>(gu_tiles_host), reinterpret_cast<const uint8_t*>(dn_tiles_host),
      S.gu_expert, S.dn_expert, E, sb + S.gu, sb + S.dn, err);
  rc = record_cuda(cudaGetLastError());
  if (rc) return rc;
  // the expert kernels in plain stream order too: the down kernel's early weight
  // prefetch (a programmatic launch) would read the staged plan before it is written
  return launch_moe_experts(act_dtype, scale_dtype, has_zeros, T, slots, H, I, group, sb + S.gu,
                            sb + S.dn, staged, rms_eps > 0.f ? (const void*)(ws + L.xn) : x,
                            ws + L.act, residual, out, err, slots, false, st);
}
