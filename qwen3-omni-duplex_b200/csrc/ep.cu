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
#include <string.h>

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
// Peer exchange (dispatch into the destinations' receive buffers, partials back into
// the owners'): when `sig` is given, the last CTA of the grid -- after every CTA fenced
// its stores at system scope and counted itself -- writes the exchange's epoch into
// flag slot `rank` of every destination; the destination waits for all slots
// (ep_wait_kernel).  Plain peer stores over NVLink (CUDA IPC mappings), no multicast.
struct PeerSignal {
  unsigned* const* flags;  // [n_ranks] each destination's flag array (slot `rank` is ours)
  unsigned* counter;       // local: CTAs done
  unsigned* epoch;         // local: exchanges done
  int rank;
};

DEVI void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

DEVI unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// the last CTA to finish signals every destination (all threads of the CTA call it)
DEVI void signal_peers(const PeerSignal& sg, int nranks) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's peer stores before its count
    const unsigned total = gridDim.x * gridDim.y;
    s_last = atomicAdd(sg.counter, 1u) == total - 1u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(sg.epoch) + 1u;
  for (int d = threadIdx.x; d < nranks; d += blockDim.x) st_release_sys(sg.flags[d] + sg.rank, e);
  __syncthreads();
  if (threadIdx.x == 0) {
    *sg.counter = 0u;  // ready for the next exchange (and graph replay)
    *sg.epoch = e;
  }
}

__global__ void __launch_bounds__(kPackThreads) ep_pack_kernel(
    const uint8_t* __restrict__ rows, int64_t row_bytes, int T, int top_k, int E, int nranks,
    int64_t ids_off, uint8_t* __restrict__ send, int32_t* __restrict__ slot_of,
    uint8_t* const* __restrict__ dst, PeerSignal sg) {
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
  // block d: this rank's block of destination d's receive buffer (peer), or of `send`
  uint8_t* blk = dst ? dst[d] + (int64_t)sg.rank * T * row_bytes : send + (int64_t)d * T * row_bytes;
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
  if (dst) signal_peers(sg, nranks);
}

// block d of `src` (n_ranks blocks of `block_bytes`) -> destination d's buffer at block
// `rank`, then the signal.  Grid (n_ranks, chunks), 16-byte copies.
__global__ void __launch_bounds__(kPackThreads) ep_put_kernel(const uint8_t* __restrict__ src,
                                                              int64_t block_bytes, int nranks,
                                                              uint8_t* const* __restrict__ dst,
                                                              PeerSignal sg) {
  const int d = blockIdx.x;
  const int64_t q16 = block_bytes >> 4;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + (int64_t)d * block_bytes);
  uint4* d4 = reinterpret_cast<uint4*>(dst[d] + (int64_t)sg.rank * block_bytes);
  for (int64_t q = (int64_t)blockIdx.y * blockDim.x + threadIdx.x; q < q16;
       q += (int64_t)gridDim.y * blockDim.x)
    d4[q] = s4[q];
  signal_peers(sg, nranks);
}

// wait until every source's flag slot holds this rank's epoch of the exchange (bounded:
// gives up after `limit` cycles with DUPLEX_DEVERR_TIMEOUT, never hangs)
__global__ void ep_wait_kernel(const unsigned* flags, const unsigned* epoch, int nranks,
                               long long limit, int* err) {
  const unsigned e = *reinterpret_cast<const volatile unsigned*>(epoch);
  for (int s = threadIdx.x; s < nranks; s += blockDim.x) {
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys(flags + s) - e) < 0) {
      if (clock64() - t0 > limit) {
        atomicOr(err, DUPLEX_DEVERR_TIMEOUT);
        break;
      }
    }
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
      reinterpret_cast<uint8_t*>(send), slot_of, nullptr, PeerSignal{});
  return record_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------- peer exchange
extern "C" int duplex_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int duplex_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return DUPLEX_ERR_ARG;
  void* p = nullptr;
  int rc = record_cuda(cudaMalloc(&p, bytes));
  if (rc) return rc;
  rc = record_cuda(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  if (!rc) rc = record_cuda(cudaIpcGetMemHandle(&h, p));
  if (rc) {
    cudaFree(p);
    return rc;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return DUPLEX_OK;
}

extern "C" int duplex_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return DUPLEX_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return record_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int duplex_ipc_close(void* ptr) { return record_cuda(cudaIpcCloseMemHandle(ptr)); }

extern "C" int duplex_ipc_free(void* ptr) { return record_cuda(cudaFree(ptr)); }

static bool valid_signal(const void* flags, const void* counter, const void* epoch, int rank,
                         int n_ranks) {
  return flags && counter && epoch && rank >= 0 && rank < n_ranks;
}

extern "C" int duplex_ep_dispatch_peer(const void* rows, int64_t row_bytes, int32_t T,
                                       int32_t top_k, int32_t E, int32_t n_ranks, int32_t rank,
                                       int64_t ids_offset, void* const* recv_peers,
                                       int32_t* slot_of, unsigned* const* flag_peers,
                                       unsigned* counter, unsigned* epoch, void* stream) {
  if (!rows || !recv_peers || !slot_of || T < 1 || T > kPackThreads || top_k < 1 || top_k > 8 ||
      n_ranks < 1 || E < n_ranks || E % n_ranks || !valid_signal(flag_peers, counter, epoch, rank, n_ranks))
    return DUPLEX_ERR_ARG;
  if ((row_bytes & 15) || ids_offset < 0 || ids_offset + 8 * (int64_t)top_k > row_bytes ||
      (reinterpret_cast<uintptr_t>(rows) & 15u) || (ids_offset & 3))
    return DUPLEX_ERR_ALIGN;
  const dim3 grid((unsigned)n_ranks, (unsigned)((T + kPackChunk - 1) / kPackChunk));
  ep_pack_kernel<<<grid, kPackThreads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(rows), row_bytes, T, top_k, E, n_ranks, ids_offset, nullptr,
      slot_of, reinterpret_cast<uint8_t* const*>(recv_peers),
      PeerSignal{flag_peers, counter, epoch, rank});
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_ep_put_peer(const void* src, int64_t block_bytes, int32_t n_ranks,
                                  int32_t rank, void* const* dst_peers, unsigned* const* flag_peers,
                                  unsigned* counter, unsigned* epoch, void* stream) {
  if (!src || !dst_peers || block_bytes < 16 || n_ranks < 1 ||
      !valid_signal(flag_peers, counter, epoch, rank, n_ranks))
    return DUPLEX_ERR_ARG;
  if ((block_bytes & 15) || (reinterpret_cast<uintptr_t>(src) & 15u)) return DUPLEX_ERR_ALIGN;
  int chunks = (int)((block_bytes / 16 + kPackThreads - 1) / kPackThreads);
  if (chunks > 64) chunks = 64;
  const dim3 grid((unsigned)n_ranks, (unsigned)chunks);
  ep_put_kernel<<<grid, kPackThreads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(src), block_bytes, n_ranks,
      reinterpret_cast<uint8_t* const*>(dst_peers), PeerSignal{flag_peers, counter, epoch, rank});
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_ep_wait(const unsigned* flags, const unsigned* epoch, int32_t n_ranks,
                              int64_t wait_limit_cycles, int32_t* err, void* stream) {
  if (!flags || !epoch || !err || n_ranks < 1) return DUPLEX_ERR_ARG;
  const long long limit = wait_limit_cycles > 0 ? wait_limit_cycles : 4000000000LL;  // ~2 s
  ep_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, epoch, n_ranks, limit, err);
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
