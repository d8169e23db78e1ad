// Expert-parallel dispatch and combine around the NCCL all-to-alls (one process per
// GPU, 128 experts split evenly over the ranks, tokens data-parallel).
//
// dispatch_pack: for every destination rank d, the exchange rows (token, its k expert
//   ids, its k weights; written by the router's top-k kernel) of this rank's tokens
//   that selected at least one of d's experts, compacted in token order into block d
//   of the send buffer.  A block has a fixed capacity of T_local rows, so the
//   all-to-all has a fixed size (no host synchronisation, graph-capturable); the rows
//   past the block's count carry ids of an expert of another rank and zero weights,
//   which the receiving expert stage skips.  slot_of[d][t] is token t's row in block d
//   (-1 when t was not sent to d).
// combine: out[t] = sum over d in rank order of the partial row that rank d returned
//   for token t (+ residual), one rounding to the activation type.
#include "common.cuh"

namespace duplex {

int record_cuda(cudaError_t e);

constexpr int kPackThreads = 512;
constexpr int kPackChunk = 8;  // tokens whose rows one CTA copies

// Grid (destination d, chunk c).  Every CTA ranks all T tokens for d (one thread per
// token, ballot + warp-count scan: cheap, and the same in every CTA of d), then copies
// the rows of tokens [c * kPackChunk, (c + 1) * kPackChunk) that go to d and writes the
// padding rows of block d with positions in the same range, so the 1-4 MB of rows of
// a layer are spread over n_ranks * T / kPackChunk CTAs.  T <= kPackThreads.
__global__ void __launch_bounds__(kPackThreads) ep_pack_kernel(
    const uint8_t* __restrict__ rows, int64_t row_bytes, int T, int top_k, int E, int nranks,
    int64_t ids_off, uint8_t* __restrict__ send, int32_t* __restrict__ slot_of) {
  __shared__ int warp_count[kPackThreads / 32];
  __shared__ int pos_s[kPackChunk];
  const int d = blockIdx.x, c0 = blockIdx.y * kPackChunk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E_l = E / nranks, e0 = d * E_l, e1 = e0 + E_l;
  bool hit = false;
  if (tid < T) {
    const int32_t* ids = reinterpret_cast<const int32_t*>(rows + (int64_t)tid * row_bytes + ids_off);
    for (int j = 0; j < top_k; ++j) hit |= ids[j] >= e0 && ids[j] < e1;
  }
  const uint32_t ballot = __ballot_sync(0xffffffffu, hit);
  if (lane == 0) warp_count[warp] = __popc(ballot);
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < kPackThreads / 32; ++w) {
    if (w < warp) before += warp_count[w];
    total += warp_count[w];
  }
  const int pos = hit ? before + __popc(ballot & ((1u << lane) - 1u)) : -1;
  if (tid >= c0 && tid < c0 + kPackChunk && tid < T) {
    pos_s[tid - c0] = pos;
    slot_of[(int64_t)d * T + tid] = pos;
  }
  __syncthreads();
  // this chunk's rows: kPackThreads / 32 / kPackChunk warps per row, 16-byte pieces
  uint8_t* blk = send + (int64_t)d * T * row_bytes;
  const int64_t q16 = row_bytes >> 4;
  constexpr int kWpr = kPackThreads / 32 / kPackChunk;
  {
    const int i = warp / kWpr, t = c0 + i;
    const int p = t < T ? pos_s[i] : -1;
    if (p >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(rows + (int64_t)t * row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(blk + (int64_t)p * row_bytes);
      for (int64_t q = (warp % kWpr) * 32 + lane; q < q16; q += 32 * kWpr) dst[q] = src[q];
    }
  }
  // padding rows with positions in this chunk's range: an expert of the next rank
  // (skipped by the receiver), weight 0
  const int sentinel = ((d + 1) % nranks) * E_l;
  const int r = c0 + tid / top_k, j = tid % top_k;
  if (tid < kPackChunk * top_k && r >= total && r < T) {
    int32_t* ids = reinterpret_cast<int32_t*>(blk + (int64_t)r * row_bytes + ids_off);
    float* w = reinterpret_cast<float*>(ids + top_k);
    ids[j] = sentinel;
    w[j] = 0.f;
  }
}

// One CTA per token: out[t][h] = sum_d part[d][slot_of[d][t]][h] (+ res[t][h]).
template <typename T>
__global__ void ep_combine_kernel(const float* __restrict__ part, const int32_t* __restrict__ slot_of,
                                  int Tn, int nranks, int H, const T* __restrict__ res,
                                  T* __restrict__ out) {
  const int t = blockIdx.x;
  for (int h4 = threadIdx.x; h4 < (H >> 2); h4 += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < nranks; ++d) {
      const int p = slot_of[(int64_t)d * Tn + t];
      if (p < 0) continue;
      const float4 v =
          reinterpret_cast<const float4*>(part + ((int64_t)d * Tn + p) * H)[h4];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    const int64_t o = (int64_t)t * H + 4 * h4;
    if (res) {
      s.x += to_f32<T>(res[o]);
      s.y += to_f32<T>(res[o + 1]);
      s.z += to_f32<T>(res[o + 2]);
      s.w += to_f32<T>(res[o + 3]);
    }
    out[o] = from_f32<T>(s.x);
    out[o + 1] = from_f32<T>(s.y);
    out[o + 2] = from_f32<T>(s.z);
    out[o + 3] = from_f32<T>(s.w);
  }
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_ep_dispatch_pack(const void* rows, int64_t row_bytes, int32_t T,
                                       int32_t top_k, int32_t E, int32_t n_ranks,
                                       int64_t ids_offset, void* send, int32_t* slot_of,
                                       void* stream) {
  if (!rows || !send || !slot_of || T < 1 || T > kPackThreads || top_k < 1 || top_k > 8 ||
      n_ranks < 1 || E < n_ranks || E % n_ranks)
    return DUPLEX_ERR_ARG;
  if ((row_bytes & 15) || ids_offset < 0 || ids_offset + 8 * (int64_t)top_k > row_bytes)
    return DUPLEX_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(send)) & 15u ||
      (ids_offset & 3))
    return DUPLEX_ERR_ALIGN;
  const dim3 grid((unsigned)n_ranks, (unsigned)((T + kPackChunk - 1) / kPackChunk));
  ep_pack_kernel<<<grid, kPackThreads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(rows), row_bytes, T, top_k, E, n_ranks, ids_offset,
      reinterpret_cast<uint8_t*>(send), slot_of);
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_ep_combine(const float* partials, const int32_t* slot_of, int32_t T,
                                 int32_t n_ranks, int32_t H, const void* residual, void* out,
                                 int act_dtype, void* stream) {
  if (!partials || !slot_of || !out || T < 1 || n_ranks < 1 || H < 4 || (H & 3))
    return DUPLEX_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(partials) & 15u)) return DUPLEX_ERR_ALIGN;
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = H / 4 < 256 ? H / 4 : 256;
  if (act_dtype == DUPLEX_DTYPE_F16)
    ep_combine_kernel<__half><<<T, threads, 0, st>>>(partials, slot_of, T, n_ranks, H,
                                                     reinterpret_cast<const __half*>(residual),
                                                     reinterpret_cast<__half*>(out));
  else if (act_dtype == DUPLEX_DTYPE_BF16)
    ep_combine_kernel<__nv_bfloat16><<<T, threads, 0, st>>>(
        partials, slot_of, T, n_ranks, H, reinterpret_cast<const __nv_bfloat16*>(residual),
        reinterpret_cast<__nv_bfloat16*>(out));
  else
    return DUPLEX_ERR_DTYPE;
  return record_cuda(cudaGetLastError());
}
