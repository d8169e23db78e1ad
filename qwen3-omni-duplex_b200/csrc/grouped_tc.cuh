// Batched-decode experts on the fifth-generation tensor cores (tcgen05), included by
// grouped.cu after its routing, bucketing and combine kernels, which this path shares.
//
// Per call: bucketing into units of at most N tokens (N = 16, 32 or 64 MMA columns),
// a gather of every unit's token rows into the MMA's shared-memory operand layout, then
// two persistent kernels (one CTA per SM) over flattened lists of (unit, 128-row tile)
// items: gate|up (128 rows = 64 gate rows and their 64 up rows, SiLU(gate) * up in the
// epilogue) and down (128 output rows, fp32 partial rows per assignment), and the shared
// combine.
//
// Weights: "tensor-core records", per (expert, 128-row tile, 128-column chunk) 8192 bytes of int4
// in a thread-per-row order, 128 scales and optionally 128 zero points (bytes).  The
// chunk is one scale group, so a thread dequantises its row's 128 values exactly as the
// reference does: (nibble - zero) is an exact small integer in the 16-bit activation
// type, times the scale is one rounding.  The values go straight into tensor memory as
// the MMA's A operand (tcgen05.st), so the 4x wider 16-bit weights never pass through
// shared memory; the MMA accumulates the tile's whole K in fp32 in tensor memory.
//
// Roles in a CTA (320 threads):
//   warps 0-3, 4-7  two dequantising warp groups, one chunk of every two-chunk stage each;
//                   thread (warp & 3) * 32 + lane owns tile row m (its tensor-memory lane);
//                   after the first chunk of the next item, the epilogue of the previous
//                   one (each group reads half of the token columns).
//   warp 8          producer: per ring stage one bulk copy of two weight chunks and one of
//                   the unit's two token tiles (16 column chunks of 8 values x N tokens each).
//   warp 9          allocates 512 tensor-memory columns; lane 0 issues the 8 MMAs
//                   (K = 16 each) of every chunk and commits them to the barriers below.
// Tensor memory: A buffers [group][3] x 64 columns at 0..383, D [2 items] x 64 at 384..511.
// Barriers: full/empty per ring stage (empty: one MMA commit per stage, which also frees
// the A buffers the stage's MMAs read); A ready (4 warps) per A buffer; D ready (commit) /
// D free (8 epilogue warps) per D buffer.  Every wait is
// bounded: on timeout the error word gets DUPLEX_DEVERR_TIMEOUT, an abort flag stops all
// roles, the MMA thread and the producer drain what they issued, and tensor memory is
// released before the CTA exits.

namespace duplex {

constexpr int kTcK = 128;                 // K per chunk (one scale group)
constexpr int kTcM = 128;                 // rows per tile (MMA M)
constexpr int kTcMaxSlots = 16;
constexpr int kTcThreads = 320;
constexpr uint32_t kTcInt4Bytes = 8192;   // 128 rows x 128 nibbles
constexpr uint32_t kTcFixed = 1024;       // barrier / flag area ahead of the ring
constexpr uint32_t kTcFull = 0, kTcEmpty = 128, kTcAReady = 256, kTcDReady = 320,
                   kTcDFree = 336, kTcDrain = 352, kTcAbort = 360, kTcTmem = 364;
constexpr int kTcABuf = 3;                // A buffers per dequantising group (64 columns each)
constexpr uint32_t kTcColsD = 384;        // first D column (after 2 x 3 A buffers)
constexpr uint32_t kTcDCols = 64;         // D columns per item (N <= 64)
constexpr int kTcCps = 2;                 // chunks per ring stage (one per dequantising group)
constexpr uint32_t kTcMinSmem = 120 * 1024;  // > half an SM: one CTA per SM, so the 512-column
                                             // tensor-memory allocation never waits

__host__ __device__ constexpr uint32_t tc_chunk_bytes(int has_zeros) {
  return kTcInt4Bytes + 256u + (has_zeros ? 128u : 0u);
}

struct TcParams {
  int E, top_k, max_units, H, I;
  int tiles, chunks;          // this kernel's weight: gate|up 2I/128 x H/128, down H/128 x I/128
  int has_zeros, ns;
  uint32_t chunk_bytes, b_bytes, stage_bytes;
  const uint8_t* rec;         // tensor-core records of local expert 0
  const uint8_t* bsrc;        // token tiles [unit][K/8][N][8 values]
  uint8_t* acm;               // gate|up output, down's token tiles [unit][I/8][N][8 values]
  const int* assign;
  const int* units;
  const int* n_units;
  float* ypart;
  int* err;
};

// Bounded wait on a phase; false (abort flag set, error recorded) on timeout or abort.
DEVI bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      set_error(err, DUPLEX_DEVERR_TIMEOUT);
      return false;
    }
  }
}

DEVI void tc_unit(const TcParams& p, int u, int N, int& e, int& first, int& n) {
  e = p.units[u * 3 + 0];
  e = (e < 0 || e >= p.E) ? 0 : e;
  first = p.units[u * 3 + 1];
  n = p.units[u * 3 + 2];
  n = n < 1 ? 1 : (n > N ? N : n);
}

// 16-bit pairs as raw words
template <typename T> struct TcPair;
template <> struct TcPair<__half> {
  static constexpr uint32_t kOff = 0x6400u;  // 1024.0: (0x6400 | n) = 1024 + n exactly
  DEVI static uint32_t sub(uint32_t a, uint32_t b) {
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  DEVI static uint32_t mul(uint32_t a, uint32_t b) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};
template <> struct TcPair<__nv_bfloat16> {
  static constexpr uint32_t kOff = 0x4300u;  // 128.0: (0x4300 | n) = 128 + n exactly
  DEVI static uint32_t sub(uint32_t a, uint32_t b) {
    const __nv_bfloat162 r =
        __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  DEVI static uint32_t mul(uint32_t a, uint32_t b) {
    const __nv_bfloat162 r =
        __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};

// Row m of the staged chunk -> tensor-memory columns ta .. ta + 63 (pairs of values).
// Record words: piece q (0..3) of row m is the 16 bytes at (q * 128 + m) * 16; word j
// (= 4 q + i) holds values 8 j .. 8 j + 7, the pair (8 j + 2 p, 8 j + 2 p + 1) in the
// nibbles at bits 4 p and 16 + 4 p.
template <typename T>
DEVI void tc_dequant(const uint8_t* stage, int m, int has_zeros, uint32_t ta) {
  const uint4* wq = reinterpret_cast<const uint4*>(stage) + m;
  const uint32_t s = reinterpret_cast<const uint16_t*>(stage + kTcInt4Bytes)[m];
  const uint32_t z = has_zeros ? (uint32_t)stage[kTcInt4Bytes + 256 + m] : 8u;
  const uint32_t z2 = (TcPair<T>::kOff + z) * 0x00010001u;
  const uint32_t s2 = s * 0x00010001u;
  const uint32_t off2 = TcPair<T>::kOff * 0x00010001u;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t r[32];
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
      const uint4 v = wq[(2 * h + qq) * 128];
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          const uint32_t t = lop3_and_or(w4[i] >> (4 * pp), 0x000F000Fu, off2);
          r[(qq * 4 + i) * 4 + pp] = TcPair<T>::mul(TcPair<T>::sub(t, z2), s2);
        }
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t rr[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) rr[k] = r[cc * 8 + k];
      tmem_st8(ta + h * 32 + cc * 8, rr);
    }
  }
}

// Producer (one thread): items [i0, i1) into the ring, two chunks per stage.  A stage is
// [weights of chunk 2 cp | of chunk 2 cp + 1 | token tile of chunk 2 cp | of 2 cp + 1]:
// both halves are contiguous at their source, so a stage costs two bulk copies (each
// copy has a fixed issue cost of a few hundred cycles, so fewer and larger copies stream
// faster).
DEVI void tc_produce(const TcParams& p, int N, uint64_t* full, uint64_t* empty, volatile int* abort_flag,
                     uint8_t* ring, int i0, int i1) {
  const uint64_t pol = policy_evict_first();
  const int pairs = p.chunks / kTcCps;
  const uint32_t wbytes = kTcCps * p.chunk_bytes, bbytes = kTcCps * p.b_bytes;
  int j = 0;
  for (int it = i0; it < i1; ++it) {
    const int u = it / p.tiles, t = it - u * p.tiles;
    int e, first, n;
    tc_unit(p, u, N, e, first, n);
    const uint8_t* wsrc = p.rec + (size_t)(e * p.tiles + t) * p.chunks * p.chunk_bytes;
    const uint8_t* bsrc = p.bsrc + (size_t)u * p.chunks * p.b_bytes;
    for (int cp = 0; cp < pairs; ++cp, ++j) {
      const int s = j % p.ns, use = j / p.ns;
      if (use > 0 && !tc_wait(&empty[s], (uint32_t)(use - 1) & 1u, abort_flag, p.err)) goto drain;
      uint8_t* dst = ring + (size_t)s * p.stage_bytes;
      mbar_arrive_expect_tx(&full[s], wbytes + bbytes);
      bulk_g2s_stream(dst, wsrc + (size_t)cp * wbytes, wbytes, &full[s], pol);
      bulk_g2s(dst + wbytes, bsrc + (size_t)cp * bbytes, bbytes, &full[s]);
    }
  }
drain:
  // no copy may still be landing when the CTA exits
  for (int k = j > p.ns ? j - p.ns : 0; k < j; ++k) {
    const long long t0 = clock64();
    while (!mbar_try_wait(&full[k % p.ns], (uint32_t)(k / p.ns) & 1u))
      if (clock64() - t0 > 200000000LL) {
        set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
        break;
      }
  }
}

// MMA issuer (one thread): the 8 K-steps of each chunk into the item's accumulator.
template <int N>
DEVI void tc_mma(const TcParams& p, uint64_t* full, uint64_t* empty, uint64_t* aready, uint64_t* dready, uint64_t* dfree, uint64_t* drain, volatile int* abort_flag, uint8_t* ring,
                 uint32_t tbase, uint32_t idesc, int i0, int i1) {
  const int pairs = p.chunks / kTcCps;
  int j = 0, ii = 0, k0 = 0, k1 = 0;  // stages so far; chunks so far of group 0 / group 1
  for (int it = i0; it < i1; ++it, ++ii) {
    const int db = ii & 1;
    const uint32_t dcol = kTcColsD + (uint32_t)db * kTcDCols;
    for (int cp = 0; cp < pairs; ++cp, ++j) {
      const int s = j % p.ns, use = j / p.ns;
      if (!tc_wait(&full[s], (uint32_t)use & 1u, abort_flag, p.err)) goto out;
      uint8_t* st = ring + (size_t)s * p.stage_bytes;
#pragma unroll
      for (int wg = 0; wg < kTcCps; ++wg) {
        const int c = cp * kTcCps + wg;
        const int k = wg ? k1++ : k0++, b = wg * kTcABuf + k % kTcABuf;
        if (!tc_wait(&aready[b], (uint32_t)(k / kTcABuf) & 1u, abort_flag, p.err)) goto out;
        if (c == 0 && ii >= 2 && !tc_wait(&dfree[db], (uint32_t)((ii >> 1) - 1) & 1u, abort_flag, p.err))
          goto out;
        tc_fence_after();
        const uint32_t acol = (uint32_t)b * 64u;
        const uint32_t b0 = smem_u32(st + kTcCps * p.chunk_bytes + (uint32_t)wg * p.b_bytes);
#pragma unroll
        for (int s8 = 0; s8 < kTcK / 16; ++s8)
          umma_ts(tbase + dcol, tbase + acol + 8u * s8, smem_desc_kmajor(b0 + (uint32_t)s8 * 32u * N, 16u * N, 128u),
                  idesc, (c | s8) != 0);
      }
      // one commit per stage (a commit costs about as much as an MMA): it frees the ring
      // slot and, for the dequantising groups, the A buffers this stage read
      umma_commit(&empty[s]);
      if (cp == pairs - 1) umma_commit(&dready[db]);
    }
  }
out:
  // every MMA this thread issued is complete before tensor memory is released
  umma_commit(drain);
  {
    const long long t0 = clock64();
    while (!mbar_try_wait(drain, 0))
      if (clock64() - t0 > 200000000LL) {
        set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
        break;
      }
  }
}

// Epilogue of the CTA's ii-th item `it` for this warp: columns [wg N/2, (wg + 1) N/2).
template <typename T, int MODE, int N>
DEVI bool tc_epilogue(const TcParams& p, uint64_t* dready, uint64_t* dfree, volatile int* abort_flag,
                      uint32_t tbase, int it, int ii) {
  constexpr int NH = N / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp >> 2, q = warp & 3, m = q * 32 + lane;
  const int db = ii & 1;
  if (!tc_wait(&dready[db], (uint32_t)(ii >> 1) & 1u, abort_flag, p.err)) return false;
  tc_fence_after();
  float y[NH];
  {
    const uint32_t ta = tmem_addr(tbase, (uint32_t)q * 32u, kTcColsD + (uint32_t)db * kTcDCols + (uint32_t)(wg * NH));
    uint32_t r[NH];
    if constexpr (NH == 8) {
      tmem_ld8(ta, r);
    } else {
#pragma unroll
      for (int h = 0; h < NH / 16; ++h) {
        uint32_t r16[16];
        tmem_ld16(ta + h * 16, r16);
#pragma unroll
        for (int k = 0; k < 16; ++k) r[h * 16 + k] = r16[k];
      }
    }
    tc_wait_ld();
#pragma unroll
    for (int k = 0; k < NH; ++k) y[k] = __uint_as_float(r[k]);
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&dfree[db]);
  const int u = it / p.tiles, t = it - u * p.tiles;
  int e, first, n;
  tc_unit(p, u, N, e, first, n);
  if constexpr (MODE == 0) {
    // lanes 0-15: gate rows, 16-31: the matching up rows (intermediate 64 t + 16 q + lane % 16)
    const int i = 64 * t + 16 * q + (lane & 15);
    T* dst = reinterpret_cast<T*>(p.acm + ((size_t)u * (p.I >> 3) + (i >> 3)) * N * 16) + (i & 7);
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const float other = __shfl_xor_sync(0xffffffffu, y[k], 16);
      const int tok = wg * NH + k;
      if (lane < 16 && tok < n) dst[(size_t)tok * 8] = from_f32<T>(silu_f32(y[k]) * other);
    }
  } else {
    const int h = t * kTcM + m;
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const int tok = wg * NH + k;
      if (tok < n) {
        const int a = p.assign[first + tok];
        p.ypart[((size_t)(a >> 3) * p.top_k + (a & 7)) * p.H + h] = y[k];
      }
    }
  }
  return true;
}

// Dequantising warp group wg: chunk wg of every stage.
template <typename T, int MODE, int N>
DEVI void tc_consume(const TcParams& p, uint64_t* full, uint64_t* empty, uint64_t* aready, uint64_t* dready,
                     uint64_t* dfree, volatile int* abort_flag, const uint8_t* ring, uint32_t tbase, int i0, int i1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp >> 2, q = warp & 3, m = q * 32 + lane;
  const int pairs = p.chunks / kTcCps;
  int j = 0, k = 0, ii = 0, pending = -1;
  for (int it = i0; it < i1; ++it, ++ii) {
    for (int cp = 0; cp < pairs; ++cp, ++j) {
      const int s = j % p.ns, use = j / p.ns, b = wg * kTcABuf + k % kTcABuf;
      if (!tc_wait(&full[s], (uint32_t)use & 1u, abort_flag, p.err)) return;
      // A buffer b was last read by stage j - kTcABuf, released with that stage's slot
      // (the slot's next release needs this group's own later A, ns > kTcABuf, so the
      // phase cannot alias)
      if (j >= kTcABuf &&
          !tc_wait(&empty[(j - kTcABuf) % p.ns], (uint32_t)((j - kTcABuf) / p.ns) & 1u, abort_flag, p.err))
        return;
      tc_dequant<T>(ring + (size_t)s * p.stage_bytes + (size_t)wg * p.chunk_bytes, m, p.has_zeros,
                    tmem_addr(tbase, (uint32_t)q * 32u, (uint32_t)b * 64u));
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aready[b]);
      ++k;
      if (pending >= 0) {  // the previous item, now that this one is under way
        if (!tc_epilogue<T, MODE, N>(p, dready, dfree, abort_flag, tbase, pending, ii - 1)) return;
        pending = -1;
      }
    }
    pending = it;
  }
  if (pending >= 0) tc_epilogue<T, MODE, N>(p, dready, dfree, abort_flag, tbase, pending, ii - 1);
}

// MODE 0: gate|up (B = gathered tokens, out = acm); MODE 1: down (B = acm, out = ypart).
template <typename T, int MODE, int N>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kTcEmpty);
  uint64_t* aready = reinterpret_cast<uint64_t*>(smem + kTcAReady);
  uint64_t* dready = reinterpret_cast<uint64_t*>(smem + kTcDReady);
  uint64_t* dfree = reinterpret_cast<uint64_t*>(smem + kTcDFree);
  uint64_t* drain = reinterpret_cast<uint64_t*>(smem + kTcDrain);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kTcAbort);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kTcTmem);
  uint8_t* ring = smem + kTcFixed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2 * kTcABuf; ++b) mbar_init(&aready[b], 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dready[b], 1);
      mbar_init(&dfree[b], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc<512>(tslot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();
  int nu = *p.n_units;
  nu = nu < 0 ? 0 : (nu > p.max_units ? p.max_units : nu);
  int i0, i1;
  g_range(nu * p.tiles, i0, i1);
  if (warp == 8) {
    if (lane == 0) tc_produce(p, N, full, empty, abort_flag, ring, i0, i1);
  } else if (warp == 9) {
    if (lane == 0)
      tc_mma<N>(p, full, empty, aready, dready, dfree, drain, abort_flag, ring, tbase,
                idesc_f16(std::is_same<T, __nv_bfloat16>::value ? 1 : 0, kTcM, N), i0, i1);
  } else {
    tc_consume<T, MODE, N>(p, full, empty, aready, dready, dfree, abort_flag, ring, tbase, i0, i1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<512>(tbase);
  }
}

// Token tiles: xcm[u][c][n][0..7] = x[token of the unit's n-th assignment][8 c .. 8 c + 7]
// for n < the unit's count (other columns are never read back).
__global__ void __launch_bounds__(256) tc_gather_kernel(const uint8_t* x, size_t x_row_bytes, const int* assign,
                                                        const int* units, const int* n_units, int max_units,
                                                        int H8, int N, uint8_t* xcm) {
  pdl_launch_dependents();
  pdl_wait();
  int nu = *n_units;
  nu = nu < 0 ? 0 : (nu > max_units ? max_units : nu);
  const long long total = (long long)nu * H8 * N;
  for (long long idx = blockIdx.x * 256ll + threadIdx.x; idx < total; idx += (long long)gridDim.x * 256) {
    const int n = (int)(idx % N);
    const long long rest = idx / N;
    const int c = (int)(rest % H8), u = (int)(rest / H8);
    const int cnt = units[u * 3 + 2];
    if (n >= cnt) continue;
    const int tok = assign[units[u * 3 + 1] + n] >> 3;
    *reinterpret_cast<uint4*>(xcm + (size_t)idx * 16) =
        __ldg(reinterpret_cast<const uint4*>(x + (size_t)tok * x_row_bytes) + c);
  }
}

// Tensor-core records from the reference's stacked tensors: packed [E][R][K/8] int32 (value k at
// bits 4 (k % 8) of word k / 8), scale [E][R][K/128], zeros [E][R][ceil(G/8)] int32 or
// null (zero point 8).  pair_halves (gate|up, R = 2 I): tile t holds intermediate rows
// 64 t .. 64 t + 63 as tile row 32 q + 16 h + j = source row h I + 64 t + 16 q + j.
template <typename S>
__global__ void tc_repack_kernel(const int32_t* __restrict__ packed, const S* __restrict__ scale,
                                 const int32_t* __restrict__ zeros, int E, int R, int K, int pair_halves,
                                 uint32_t chunk_bytes, uint32_t* __restrict__ out) {
  const int C = K / 8, G = K / kTcK, GZ = (G + 7) / 8, tiles = R / kTcM;
  const uint32_t wpc = chunk_bytes / 4u;
  const long long total = (long long)E * tiles * G * wpc;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long ch = idx / wpc;
    const uint32_t o = (uint32_t)(idx - ch * wpc) * 4u;
    const int c = (int)(ch % G);
    const long long et = ch / G;
    const int t = (int)(et % tiles), e = (int)(et / tiles);
    auto src_row = [&](int mm) {
      if (!pair_halves) return t * kTcM + mm;
      const int qq = mm >> 5, hh = (mm >> 4) & 1, jj = mm & 15;
      return hh * (R / 2) + 64 * t + 16 * qq + jj;
    };
    uint32_t val = 0;
    if (o < kTcInt4Bytes) {
      const int qd = (int)(o >> 11), mm = (int)((o >> 4) & 127u), wi = (int)((o >> 2) & 3u);
      const int jw = 4 * qd + wi;
      const uint32_t w = (uint32_t)packed[((long long)e * R + src_row(mm)) * C + 16 * c + jw];
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        val |= ((w >> (8 * pp)) & 15u) << (4 * pp);
        val |= ((w >> (8 * pp + 4)) & 15u) << (16 + 4 * pp);
      }
    } else if (o < kTcInt4Bytes + 256u) {
      const int m0 = (int)((o - kTcInt4Bytes) >> 1);
      const uint16_t a = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * R + src_row(m0)) * G + c]);
      const uint16_t b = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * R + src_row(m0 + 1)) * G + c]);
      val = (uint32_t)a | ((uint32_t)b << 16);
    } else {
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const int mm = (int)(o - kTcInt4Bytes - 256u) + bb;
        const uint32_t z = ((uint32_t)zeros[((long long)e * R + src_row(mm)) * GZ + (c >> 3)] >> ((c & 7) * 4)) & 15u;
        val |= z << (8 * bb);
      }
    }
    out[idx] = val;
  }
}

// ---------------------------------------------------------------------- host side
static bool tc_geometry_ok(int H, int I, int group) {  // whole stages of two chunks
  return group == kTcK && H % (kTcCps * kTcK) == 0 && I % (kTcCps * kTcK) == 0;
}

// MMA columns (the unit token cap) for T tokens: units of at most N tokens.
static int tc_cols(int T, int E_total, int top_k) {
  const int tk = T * top_k;
  if (tk <= 8 * E_total) return 16;
  if (tk <= 20 * E_total) return 32;
  return 64;
}

struct TcScratch {
  GScratch g;
  size_t xcm, acm;
};

static TcScratch tc_scratch(int T, int E, int H, int I, int top_k, int N) {
  TcScratch s;
  size_t off = 0;
  s.g.max_units = E + (T * top_k + N - 1) / N + 1;
  s.g.logits = off; off += align_up((size_t)T * E * 4, 256);
  s.g.sel = off; off += align_up((size_t)T * top_k * 4, 256);
  s.g.w = off; off += align_up((size_t)T * top_k * 4, 256);
  s.g.assign = off; off += align_up((size_t)T * top_k * 4, 256);
  s.g.units = off; off += align_up((size_t)s.g.max_units * 12, 256);
  s.g.n_units = off; off += 256;
  s.g.act = off;  // unused here
  s.g.ypart = off; off += align_up((size_t)T * top_k * H * 4, 256);
  s.xcm = off; off += align_up((size_t)s.g.max_units * H * N * 2, 256);
  s.acm = off; off += align_up((size_t)s.g.max_units * I * N * 2, 256);
  s.g.total = off;
  return s;
}

static void tc_ring(int N, int has_zeros, TcParams& p) {
  p.chunk_bytes = tc_chunk_bytes(has_zeros);
  p.b_bytes = 16u * (uint32_t)N * 16u;
  p.stage_bytes = (uint32_t)align_up((size_t)kTcCps * (p.chunk_bytes + p.b_bytes), 128);
  int ns = (int)((kGSmemMax - kTcFixed) / p.stage_bytes);
  p.ns = ns > kTcMaxSlots ? kTcMaxSlots : ns;
}

static uint32_t tc_smem(const TcParams& p) {
  const uint32_t s = kTcFixed + (uint32_t)p.ns * p.stage_bytes;
  return s < kTcMinSmem ? kTcMinSmem : s;
}

template <typename T, int MODE>
static void (*tc_kernel(int N))(TcParams) {
  if (N == 16) return tc_expert_kernel<T, MODE, 16>;
  if (N == 32) return tc_expert_kernel<T, MODE, 32>;
  return tc_expert_kernel<T, MODE, 64>;
}

static int tc_expert_stage(const void* x, size_t x_row_bytes, bool f16, int T, const int* sel, const float* w,
                           int meta_stride, int top_k, int e_begin, int E, int E_total, int H, int I, int has_zeros,
                           const void* gu_rec, const void* dn_rec, const TcScratch& L, int N, uint8_t* ws,
                           const void* residual, void* out, int out_f32, int* err, cudaStream_t st, bool pdl_first) {
  int rc;
  const GScratch& G = L.g;
  {
    const int NA = T * top_k, nch = (NA + 31) / 32;
    const int smem = (int)(align_up((size_t)nch * E, 16) + align_up((size_t)nch * E * 2, 16) +
                           3 * kMaxExperts * 4 + 16 * 4 + (size_t)NA * 4);
    if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(g_bucket_kernel), kGSmemMax))) return rc;
    if ((rc = g_launch(g_bucket_kernel, dim3(1), dim3(512), smem, st, pdl_first, sel, meta_stride, T, E, top_k, N,
                       e_begin, E_total, reinterpret_cast<int*>(ws + G.assign), reinterpret_cast<int*>(ws + G.units),
                       reinterpret_cast<int*>(ws + G.n_units), G.max_units, err)))
      return rc;
  }
  const int* assign = reinterpret_cast<const int*>(ws + G.assign);
  const int* units = reinterpret_cast<const int*>(ws + G.units);
  const int* n_units = reinterpret_cast<const int*>(ws + G.n_units);
  const int nsm = num_sms();
  if ((rc = g_launch(tc_gather_kernel, dim3(nsm * 4), dim3(256), 0, st, true, reinterpret_cast<const uint8_t*>(x),
                     x_row_bytes, assign, units, n_units, G.max_units, H / 8, N, ws + L.xcm)))
    return rc;
  TcParams p = {};
  p.E = E; p.top_k = top_k; p.max_units = G.max_units; p.H = H; p.I = I; p.has_zeros = has_zeros;
  p.assign = assign; p.units = units; p.n_units = n_units;
  p.ypart = reinterpret_cast<float*>(ws + G.ypart);
  p.acm = ws + L.acm;
  p.err = err;
  tc_ring(N, has_zeros, p);
  if (p.ns <= kTcABuf) return DUPLEX_ERR_UNSUPPORTED;  // A-buffer release needs ns > kTcABuf
  // gate|up
  p.tiles = 2 * I / kTcM; p.chunks = H / kTcK;
  p.rec = reinterpret_cast<const uint8_t*>(gu_rec);
  p.bsrc = ws + L.xcm;
  void (*ka)(TcParams) = f16 ? tc_kernel<__half, 0>(N) : tc_kernel<__nv_bfloat16, 0>(N);
  if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(ka), kGSmemMax))) return rc;
  if ((rc = g_launch(ka, dim3(nsm), dim3(kTcThreads), tc_smem(p), st, true, p))) return rc;
  // down
  p.tiles = H / kTcM; p.chunks = I / kTcK;
  p.rec = reinterpret_cast<const uint8_t*>(dn_rec);
  p.bsrc = ws + L.acm;
  void (*kd)(TcParams) = f16 ? tc_kernel<__half, 1>(N) : tc_kernel<__nv_bfloat16, 1>(N);
  if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(kd), kGSmemMax))) return rc;
  if ((rc = g_launch(kd, dim3(nsm), dim3(kTcThreads), tc_smem(p), st, true, p))) return rc;
  // combine
  const float* yp = reinterpret_cast<const float*>(ws + G.ypart);
  const unsigned blocks = (unsigned)(((size_t)T * H / 4 + 255) / 256);
  const dim3 cg(blocks), cb(256);
  if (f16) {
    const __half* res = reinterpret_cast<const __half*>(residual);
    if (out_f32)
      return g_launch(g_combine_kernel<__half, float>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res,
                      T, H, top_k, reinterpret_cast<float*>(out));
    return g_launch(g_combine_kernel<__half, __half>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E, res,
                    T, H, top_k, reinterpret_cast<__half*>(out));
  }
  const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(residual);
  if (out_f32)
    return g_launch(g_combine_kernel<__nv_bfloat16, float>, cg, cb, 0, st, true, yp, w, sel, meta_stride, e_begin, E,
                    res, T, H, top_k, reinterpret_cast<float*>(out));
  return g_launch(g_combine_kernel<__nv_bfloat16, __nv_bfloat16>, cg, cb, 0, st, true, yp, w, sel, meta_stride,
                  e_begin, E, res, T, H, top_k, reinterpret_cast<__nv_bfloat16*>(out));
}

}  // namespace duplex
