// int4 dequant-GEMV family for batch <= 8 on sm_100a.
//
// One persistent CTA per SM = 8 consumer warps + 1 producer warp.
//
// Producer: streams "stages" = 16 weight rows x full K of one expert, straight
// from the reference's packed layout [E][Rs][K/8] int32 (rows are contiguous
// K/2 bytes), plus the 16 rows' group scales and zero points, with 1-D bulk
// copies (cp.async.bulk, no multicast) into a ring of shared-memory stages.
// Weight rows land at a pitch of an odd number of 16-byte units so ldmatrix
// reads of 8 rows hit 8 distinct bank groups.  Weights never exist in a
// dequantised form outside registers.
//
// Consumers: every consumer warp owns a fixed slice of the K windows (32
// columns each) of every stage (split-K).  Per window: one ldmatrix.x2 gives the
// lane the packed word of row g and row g+8, the nibbles become exact 16-bit
// (n - z) integers in registers (Dq<T>), and two m16n8k16 MMAs multiply them by
// the activations, whose 8 batch rows are the MMA's N dimension.  Group scales
// are applied in fp32 when the group changes.  Partial sums of the 8 warps are
// reduced through shared memory once per output tile.
//
// Modes (template):
//   kPlain  : out[j][r] fp32 = W[sel[j]] . x_j           (dequant_gemv)
//   kLinear : dense rows, bias / residual epilogue       (TritonPackedLinear)
//   kGateUp : unit u rows [rb] and [I+rb] -> act = silu(gate) * up   (MoE)
//   kDown   : all units of one row block, routing-weighted combine   (MoE)
//
// PDL: kLinear/kDown issue their weight copies before griddepcontrol.wait (the
// weights do not depend on the previous kernel); kDown reads the routing plan
// before the wait because the gate|up kernel only triggers its dependents after
// its own wait on the router has returned.
#include "common.cuh"
#include "moe.cuh"

namespace duplex {

constexpr int kCW = 8;  // consumer warps
constexpr int kConsumers = kCW * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kStagesMax = 16;

enum : int { kPlain = 0, kLinear = 1, kGateUp = 2, kDown = 3 };

// fixed shared-memory map (bytes)
constexpr uint32_t kOffFull = 0;       // kStagesMax mbarriers
constexpr uint32_t kOffEmpty = 128;    // kStagesMax mbarriers
constexpr uint32_t kOffAbort = 256;    // int
constexpr uint32_t kOffXslot = 320;    // kStagesMax ints (producer bookkeeping)
constexpr uint32_t kOffUnitW = 512;    // kMaxUnits * kMaxTokens floats (2048 B)
constexpr uint32_t kOffRed = 2560;     // kCW * 8 * 32 floats (8192 B)
constexpr uint32_t kOffXsh = 10752;    // shared activations, then the stage ring

struct GemvParams {
  const int32_t* packed;
  const void* scale;
  const int32_t* zeros;
  int E, R, Rs, K, G, GZ, group;
  const void* x;
  long long x_col_stride;   // elements between batch columns
  long long x_slot_stride;  // elements between slots / units (per-stage activations)
  int ncols;
  const int32_t* sel;
  int nslots;
  const MoePlan* plan;
  int I;
  void* out;
  long long out_slot_stride, out_col_stride;
  const void* bias;
  const void* residual;
  long long res_col_stride;
  int* err;
  int nstages;
  uint32_t row_pitch, off_scale, off_zero, off_x, stage_bytes, x_pitch;
  uint32_t wbytes, sbytes, zbytes, xbytes_row;
  uint32_t smem_stage0;
  int prefetch;
  int x_per_stage;
  float rms_eps;            // > 0: RMS-normalise the shared activation rows on load
};

template <int MODE>
DEVI int tiles_of(const GemvParams& p, int n_units, int Rb) {
  if (MODE == kPlain) return p.nslots * Rb;
  if (MODE == kLinear) return Rb;
  if (MODE == kGateUp) return n_units * (p.I >> 4);
  return Rb;  // kDown
}

template <int MODE>
DEVI int stages_of(int n_units) {
  return MODE == kGateUp ? 2 : (MODE == kDown ? n_units : 1);
}

// stage -> (expert, row block, activation slot)
template <int MODE>
DEVI void stage_decode(const GemvParams& p, int tile, int s, int Rb, int& expert, int& rb,
                       int& xs) {
  if (MODE == kPlain) {
    const int slot = tile / Rb;
    rb = tile - slot * Rb;
    expert = p.sel[slot];
    xs = slot;
  } else if (MODE == kLinear) {
    expert = 0;
    rb = tile;
    xs = 0;
  } else if (MODE == kGateUp) {
    const int per = p.I >> 4;
    const int u = tile / per;
    rb = (tile - u * per) + s * per;
    expert = p.plan->unit_expert[u];
    xs = u;
  } else {
    rb = tile;
    expert = p.plan->unit_expert[s];
    xs = s;
  }
}

DEVI bool wait_limited(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

template <typename T, typename S, int MODE>
__global__ void __launch_bounds__(kThreads, 2) dq_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  int* xslot_of = reinterpret_cast<int*>(smem + kOffXslot);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nstages;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], kCW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (MODE != kGateUp) pdl_launch_dependents();

  const int Rb = (p.R + 15) >> 4;

  if (warp == kCW) {
    // ------------------------------------------------------------ producer warp
    const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(p.packed);
    const uint8_t* ssrc = reinterpret_cast<const uint8_t*>(p.scale);
    const uint8_t* zsrc = reinterpret_cast<const uint8_t*>(p.zeros);
    const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(p.x);
    const uint64_t pol = policy_evict_first();
    bool waited = false;
    if (!p.prefetch) {
      pdl_wait();
      waited = true;
      if (MODE == kGateUp) pdl_launch_dependents();
    }
    int n_units = 0;
    if (MODE == kGateUp || MODE == kDown) {
      n_units = p.plan->n_units;
      n_units = n_units < 0 ? 0 : (n_units > kMaxUnits ? kMaxUnits : n_units);
    }
    const int ntiles = tiles_of<MODE>(p, n_units, Rb);
    const int nst = stages_of<MODE>(n_units);

    auto issue_x = [&](int j) {
      const int slot = j % NS;
      if (p.x_per_stage) {
        const int xs = xslot_of[slot];
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)p.ncols * p.xbytes_row);
        __syncwarp();
        if (lane < p.ncols) {
          const uint8_t* src =
              xsrc + ((long long)xs * p.x_slot_stride + (long long)lane * p.x_col_stride) * 2;
          bulk_g2s(smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes + p.off_x +
                       (uint32_t)lane * p.x_pitch,
                   src, p.xbytes_row, &full[slot]);
        }
        __syncwarp();
      } else {
        if (lane == 0) mbar_arrive(&full[slot]);
        __syncwarp();
      }
    };

    int i = 0, xi = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      for (int s = 0; s < nst; ++s, ++i) {
        const int slot = i % NS;
        if (i >= NS) {
          if (!waited) {
            pdl_wait();
            waited = true;
            for (; xi < i; ++xi) issue_x(xi);
          }
          if (!mbar_wait_bounded(&empty[slot], (uint32_t)((i / NS) - 1) & 1u, abort_flag)) {
            if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
          }
        }
        int expert, rb, xs;
        stage_decode<MODE>(p, tile, s, Rb, expert, rb, xs);
        if ((unsigned)expert >= (unsigned)p.E) {
          if (lane == 0) set_error(p.err, DUPLEX_DEVERR_EXPERT);
          expert = 0;
        }
        if (lane == 0) xslot_of[slot] = xs;
        uint8_t* st = smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes;
        const size_t row0 = (size_t)expert * (size_t)p.Rs + (size_t)rb * 16u;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], 16u * p.wbytes + p.sbytes + p.zbytes);
        __syncwarp();
        if (lane < 16) {
          bulk_g2s_stream(st + (uint32_t)lane * p.row_pitch, wsrc + (row0 + lane) * p.wbytes,
                          p.wbytes, &full[slot], pol);
        } else if (lane == 16) {
          bulk_g2s_stream(st + p.off_scale, ssrc + row0 * (size_t)p.G * 2u, p.sbytes, &full[slot],
                          pol);
        } else if (lane == 17 && p.zbytes) {
          bulk_g2s_stream(st + p.off_zero, zsrc + row0 * (size_t)p.GZ * 4u, p.zbytes, &full[slot],
                          pol);
        }
        __syncwarp();
        if (waited) {
          issue_x(i);
          xi = i + 1;
        }
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
      for (; xi < i; ++xi) issue_x(xi);
    }
    // drain: never leave the CTA while a bulk copy may still target its smem
    if (lane == 0) {
      const int first = i > NS ? i - NS : 0;
      for (int j = first; j < i; ++j) {
        if (!wait_limited(&full[j % NS], (uint32_t)(j / NS) & 1u, 200000000LL)) {
          set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
          break;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  pdl_wait();
  if (MODE == kGateUp) pdl_launch_dependents();
  const int g = lane >> 2, t = lane & 3;
  uint8_t* xsh = smem + kOffXsh;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* unit_w = reinterpret_cast<float*>(smem + kOffUnitW);

  int n_units = 0;
  if (MODE == kGateUp || MODE == kDown) {
    n_units = p.plan->n_units;
    n_units = n_units < 0 ? 0 : (n_units > kMaxUnits ? kMaxUnits : n_units);
  }
  if (!p.x_per_stage) {
    const int per_row = p.K >> 3;  // 16-byte chunks per activation row
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(p.x);
    for (int idx = tid; idx < p.ncols * per_row; idx += kConsumers) {
      const int n = idx / per_row, c = idx - n * per_row;
      const uint4 v =
          *reinterpret_cast<const uint4*>(xb + ((size_t)n * p.x_col_stride + (size_t)c * 8) * 2);
      *reinterpret_cast<uint4*>(xsh + (uint32_t)n * p.x_pitch + (uint32_t)c * 16) = v;
    }
  }
  if (MODE == kDown) {
    for (int idx = tid; idx < n_units * kMaxTokens; idx += kConsumers) unit_w[idx] = p.plan->unit_w[idx];
  }
  named_bar_sync(1, kConsumers);
  if (!p.x_per_stage && p.rms_eps > 0.f) {
    // y = round(x * rsqrt(mean(x^2) + eps)) per activation row (weightless RMSNorm)
    float ss[kMaxTokens];
#pragma unroll
    for (int n = 0; n < kMaxTokens; ++n) {
      float a = 0.f;
      if (n < p.ncols) {
        const T* row = reinterpret_cast<const T*>(xsh + (uint32_t)n * p.x_pitch);
        for (int c = tid; c < p.K; c += kConsumers) {
          const float v = to_f32<T>(row[c]);
          a = fmaf(v, v, a);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      ss[n] = a;
    }
    if (lane == 0) {
#pragma unroll
      for (int n = 0; n < kMaxTokens; ++n) red[warp * kMaxTokens + n] = ss[n];
    }
    named_bar_sync(1, kConsumers);
    for (int n = 0; n < p.ncols; ++n) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) tot += red[w * kMaxTokens + n];
      const float inv = 1.0f / sqrtf(tot / (float)p.K + p.rms_eps);
      T* row = reinterpret_cast<T*>(xsh + (uint32_t)n * p.x_pitch);
      for (int c = tid; c < p.K; c += kConsumers) row[c] = from_f32<T>(to_f32<T>(row[c]) * inv);
    }
    named_bar_sync(1, kConsumers);
  }

  const int ntiles = tiles_of<MODE>(p, n_units, Rb);
  const int nst = stages_of<MODE>(n_units);
  const int nW = p.K >> 5;
  const int wbeg = (warp * nW) / kCW, wend = ((warp + 1) * nW) / kCW;
  const bool xon = g < p.ncols;

  int i = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = 0.f;

    for (int s = 0; s < nst; ++s, ++i) {
      const int slot = i % NS;
      if (!mbar_wait_bounded(&full[slot], (uint32_t)(i / NS) & 1u, abort_flag)) {
        if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
      }
      const uint8_t* st = smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes;
      const uint8_t* xs = p.x_per_stage ? st + p.off_x : xsh;
      const S* sc = reinterpret_cast<const S*>(st + p.off_scale);
      const uint32_t* zw = reinterpret_cast<const uint32_t*>(st + p.off_zero);
      const uint32_t wrow = smem_u32(st) + (uint32_t)(lane & 15) * p.row_pitch;
      const uint8_t* xrow = xs + (uint32_t)g * p.x_pitch + (uint32_t)t * 16;

      float part[4] = {0.f, 0.f, 0.f, 0.f};
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
      int cur = -1;
      float sa = 0.f, sb = 0.f;
      uint32_t loa = 0, hia = 0, lob = 0, hib = 0;
      for (int win = wbeg; win < wend; ++win) {
        const int grp = (win << 5) / p.group;
        if (grp != cur) {
          if (cur >= 0) {
            sacc[0] += sa * part[0];
            sacc[1] += sa * part[1];
            sacc[2] += sb * part[2];
            sacc[3] += sb * part[3];
            part[0] = part[1] = part[2] = part[3] = 0.f;
          }
          cur = grp;
          sa = to_f32<S>(sc[g * p.G + grp]);
          sb = to_f32<S>(sc[(g + 8) * p.G + grp]);
          uint32_t za = 8u, zb = 8u;
          if (p.zbytes) {
            const int sh = (grp & 7) * 4;
            za = (zw[g * p.GZ + (grp >> 3)] >> sh) & 0xFu;
            zb = (zw[(g + 8) * p.GZ + (grp >> 3)] >> sh) & 0xFu;
          }
          Dq<T>::consts(za, loa, hia);
          Dq<T>::consts(zb, lob, hib);
        }
        uint32_t wa, wb;
        ldsm_x2(wa, wb, wrow + (uint32_t)win * 16u);
        uint32_t xa0 = 0, xa1 = 0, xb0 = 0, xb1 = 0;
        if (xon) {
          const uint4 v = *reinterpret_cast<const uint4*>(xrow + (uint32_t)win * 64u);
          x_frags(v, xa0, xa1, xb0, xb1);
        }
        uint32_t A[4], B[4];
        Dq<T>::expand(wa, wb, loa, hia, lob, hib, A, B);
        MmaOp<T>::run(part, A[0], A[1], A[2], A[3], xa0, xa1);
        MmaOp<T>::run(part, B[0], B[1], B[2], B[3], xb0, xb1);
      }
      if (cur >= 0) {
        sacc[0] += sa * part[0];
        sacc[1] += sa * part[1];
        sacc[2] += sb * part[2];
        sacc[3] += sb * part[3];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);

      if (MODE == kGateUp) {
        const int o = s * 4;
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[o + r] = sacc[r];
      } else if (MODE == kDown) {
        const float w0 = unit_w[s * kMaxTokens + 2 * t];
        const float w1 = unit_w[s * kMaxTokens + 2 * t + 1];
        acc[0] += w0 * sacc[0];
        acc[1] += w1 * sacc[1];
        acc[2] += w0 * sacc[2];
        acc[3] += w1 * sacc[3];
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] += sacc[r];
      }
    }

    // ---- split-K reduction across the 8 consumer warps, then the epilogue
    constexpr int NREG = (MODE == kGateUp) ? 8 : 4;
#pragma unroll
    for (int r = 0; r < NREG; ++r) red[(warp * 8 + r) * 32 + lane] = acc[r];
    named_bar_sync(1, kConsumers);
    if (tid < 128) {
      const int n = tid >> 4, r = tid & 15;
      const int gl = (r & 7) * 4 + (n >> 1);
      const int ri = (r >> 3) * 2 + (n & 1);
      float v = 0.f, v2 = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) {
        v += red[(w * 8 + ri) * 32 + gl];
        if (MODE == kGateUp) v2 += red[(w * 8 + 4 + ri) * 32 + gl];
      }
      if (MODE == kPlain) {
        const int slot = tile / Rb;
        const int row = (tile - slot * Rb) * 16 + r;
        if (n < p.ncols && row < p.R)
          reinterpret_cast<float*>(p.out)[slot * p.out_slot_stride + n * p.out_col_stride + row] = v;
      } else if (MODE == kLinear) {
        const int row = tile * 16 + r;
        if (n < p.ncols && row < p.R) {
          T y = from_f32<T>(v);
          if (p.bias) y = from_f32<T>(to_f32<T>(y) + to_f32<T>(reinterpret_cast<const T*>(p.bias)[row]));
          if (p.residual)
            y = from_f32<T>(to_f32<T>(y) +
                            to_f32<T>(reinterpret_cast<const T*>(p.residual)[n * p.res_col_stride + row]));
          reinterpret_cast<T*>(p.out)[n * p.out_col_stride + row] = y;
        }
      } else if (MODE == kGateUp) {
        const int per = p.I >> 4;
        const int u = tile / per;
        const int row = (tile - u * per) * 16 + r;
        if (n < p.ncols) {
          const uint32_t mask = p.plan->unit_mask[u];
          const float a = ((mask >> n) & 1u) ? silu_f32(v) * v2 : 0.f;
          reinterpret_cast<T*>(p.out)[((size_t)u * kMaxTokens + n) * p.I + row] = from_f32<T>(a);
        }
      } else {
        const int row = tile * 16 + r;
        if (n < p.ncols && row < p.R) {
          float y = v;
          if (p.residual)
            y += to_f32<T>(reinterpret_cast<const T*>(p.residual)[n * p.res_col_stride + row]);
          reinterpret_cast<T*>(p.out)[n * p.out_col_stride + row] = from_f32<T>(y);
        }
      }
    }
    named_bar_sync(1, kConsumers);
  }
}

// ====================================================================== host side
static int g_num_sms = 0;
static int g_last_cuda = 0;

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms = n > 0 ? n : 148;
  }
  return g_num_sms;
}

int record_cuda(cudaError_t e) {
  if (e == cudaSuccess) return DUPLEX_OK;
  g_last_cuda = (int)e;
  return DUPLEX_ERR_CUDA;
}

int last_cuda_error() { return g_last_cuda; }

static inline uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

constexpr size_t kDefaultSmemBudget = 112 * 1024;
constexpr size_t kMaxSmem = 227 * 1024;

// Fill the shared-memory geometry of `p`; returns the dynamic smem bytes or 0.
static size_t plan_geometry(GemvParams& p, bool has_zeros, size_t budget) {
  p.G = (p.K + p.group - 1) / p.group;
  p.GZ = (p.G + 7) / 8;
  p.wbytes = (uint32_t)p.K / 2u;
  uint32_t P = up(p.wbytes, 16);
  if (((P >> 4) & 1u) == 0) P += 16;
  p.row_pitch = P;
  p.sbytes = 16u * (uint32_t)p.G * 2u;
  p.zbytes = has_zeros ? 16u * (uint32_t)p.GZ * 4u : 0u;
  p.off_scale = 16u * P;
  p.off_zero = p.off_scale + up(p.sbytes, 16);
  p.x_pitch = up((uint32_t)p.K * 2u, 128) + 64u;
  p.off_x = up(p.off_zero + p.zbytes, 128);
  p.xbytes_row = (uint32_t)p.K * 2u;
  const uint32_t sb = p.off_x + (p.x_per_stage ? (uint32_t)p.ncols * p.x_pitch : 0u);
  p.stage_bytes = up(sb, 128);
  p.smem_stage0 = up(kOffXsh + (p.x_per_stage ? 0u : (uint32_t)p.ncols * p.x_pitch), 128);
  size_t b = budget;
  int ns = (int)((b > p.smem_stage0 ? b - p.smem_stage0 : 0) / p.stage_bytes);
  if (ns < 2) {
    b = kMaxSmem;
    ns = (int)((b - p.smem_stage0) / p.stage_bytes);
  }
  if (ns < 2) return 0;
  if (ns > kStagesMax) ns = kStagesMax;
  p.nstages = ns;
  return (size_t)p.smem_stage0 + (size_t)ns * p.stage_bytes;
}

template <typename T, typename S, int MODE>
static int launch(GemvParams& p, int grid, size_t smem, bool pdl, cudaStream_t stream) {
  auto kern = dq_gemv_kernel<T, S, MODE>;
  static size_t configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return record_cuda(e);
    configured = kMaxSmem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, p));
}

template <int MODE>
static int dispatch(int act_dtype, int scale_dtype, GemvParams& p, int grid, size_t smem, bool pdl,
                    cudaStream_t st) {
  if (act_dtype == DUPLEX_DTYPE_F16 && scale_dtype == DUPLEX_DTYPE_F16)
    return launch<__half, __half, MODE>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_F16 && scale_dtype == DUPLEX_DTYPE_BF16)
    return launch<__half, __nv_bfloat16, MODE>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_BF16 && scale_dtype == DUPLEX_DTYPE_BF16)
    return launch<__nv_bfloat16, __nv_bfloat16, MODE>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_BF16 && scale_dtype == DUPLEX_DTYPE_F16)
    return launch<__nv_bfloat16, __half, MODE>(p, grid, smem, pdl, st);
  return DUPLEX_ERR_DTYPE;
}

static inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int check_weights(const int32_t* packed, const void* scale, const int32_t* zeros,
                         int scale_dtype, int E, int R, int Rs, int K, int group) {
  if (!packed || !scale) return DUPLEX_ERR_ARG;
  if (E < 1 || R < 1 || Rs < R || K < 32 || group < 32) return DUPLEX_ERR_ARG;
  if (scale_dtype != DUPLEX_DTYPE_F16 && scale_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if ((Rs & 15) || (K & 31) || (group & 31)) return DUPLEX_ERR_UNSUPPORTED;
  if (!al16(packed) || !al16(scale) || (zeros && !al16(zeros))) return DUPLEX_ERR_ALIGN;
  return DUPLEX_OK;
}

struct MoeLaunch;  // fwd

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_dq_gemv(const void* x, int act_dtype, int64_t x_slot_stride,
                              const int32_t* packed, const void* scale, const int32_t* zeros,
                              int scale_dtype, int32_t E, int32_t R, int32_t Rs, int32_t K,
                              int32_t group, const int32_t* sel, int32_t nsel, float* out,
                              int32_t* err, void* stream) {
  int rc = check_weights(packed, scale, zeros, scale_dtype, E, R, Rs, K, group);
  if (rc) return rc;
  if (!x || !sel || !out || nsel < 1) return DUPLEX_ERR_ARG;
  if (!al16(x) || (x_slot_stride & 7)) return DUPLEX_ERR_ALIGN;
  GemvParams p = {};
  p.packed = packed; p.scale = scale; p.zeros = zeros;
  p.E = E; p.R = R; p.Rs = Rs; p.K = K; p.group = group;
  p.x = x; p.x_col_stride = 0; p.x_slot_stride = x_slot_stride; p.ncols = 1;
  p.sel = sel; p.nslots = nsel;
  p.out = out; p.out_slot_stride = R; p.out_col_stride = 0;
  p.err = err;
  p.prefetch = 0;
  p.x_per_stage = x_slot_stride != 0;
  const size_t smem = plan_geometry(p, zeros != nullptr, kDefaultSmemBudget);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  const int tiles = nsel * ((R + 15) / 16);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return dispatch<kPlain>(act_dtype, scale_dtype, p, grid, smem, false, (cudaStream_t)stream);
}

extern "C" int duplex_packed_linear(const void* x, int act_dtype, int32_t B, int64_t x_row_stride,
                                    const int32_t* packed, const void* scale, const int32_t* zeros,
                                    int scale_dtype, int32_t R, int32_t Rs, int32_t K, int32_t group,
                                    const void* bias, const void* residual, int64_t res_row_stride,
                                    void* out, int64_t out_row_stride, float rms_eps, int pdl,
                                    void* stream) {
  int rc = check_weights(packed, scale, zeros, scale_dtype, 1, R, Rs, K, group);
  if (rc) return rc;
  if (!x || !out || B < 1 || B > kMaxTokens) return DUPLEX_ERR_ARG;
  if (!al16(x) || (x_row_stride & 7)) return DUPLEX_ERR_ALIGN;
  GemvParams p = {};
  p.packed = packed; p.scale = scale; p.zeros = zeros;
  p.E = 1; p.R = R; p.Rs = Rs; p.K = K; p.group = group;
  p.x = x; p.x_col_stride = x_row_stride; p.x_slot_stride = 0; p.ncols = B;
  p.out = out; p.out_slot_stride = 0; p.out_col_stride = out_row_stride;
  p.bias = bias; p.residual = residual; p.res_col_stride = res_row_stride;
  p.prefetch = pdl ? 1 : 0;
  p.x_per_stage = 0;
  p.rms_eps = rms_eps;
  const size_t smem = plan_geometry(p, zeros != nullptr, kDefaultSmemBudget);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  const int tiles = (R + 15) / 16;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return dispatch<kLinear>(act_dtype, scale_dtype, p, grid, smem, pdl != 0, (cudaStream_t)stream);
}

namespace duplex {

// Gate|up and down launches of the decode MoE (T <= 8); called by moe.cu.
int launch_moe_experts(int act_dtype, int scale_dtype, int T, int E, int H, int I, int group,
                       const int32_t* gu_packed, const void* gu_scale, const int32_t* gu_zeros,
                       const int32_t* dn_packed, const void* dn_scale, const int32_t* dn_zeros,
                       const MoePlan* plan, const void* x, void* act, const void* residual,
                       void* out, int* err, int max_units, bool pdl, cudaStream_t st) {
  int rc = check_weights(gu_packed, gu_scale, gu_zeros, scale_dtype, E, 2 * I, 2 * I, H, group);
  if (rc) return rc;
  rc = check_weights(dn_packed, dn_scale, dn_zeros, scale_dtype, E, H, H, I, group);
  if (rc) return rc;
  if ((I & 15) || (H & 15)) return DUPLEX_ERR_UNSUPPORTED;

  GemvParams a = {};
  a.packed = gu_packed; a.scale = gu_scale; a.zeros = gu_zeros;
  a.E = E; a.R = 2 * I; a.Rs = 2 * I; a.K = H; a.group = group;
  a.x = x; a.x_col_stride = H; a.x_slot_stride = 0; a.ncols = T;
  a.plan = plan; a.I = I;
  a.out = act;
  a.err = err;
  a.prefetch = 0;
  a.x_per_stage = 0;
  size_t smem = plan_geometry(a, gu_zeros != nullptr, kDefaultSmemBudget);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  int tiles = max_units * (I / 16);
  int grid = tiles < num_sms() ? tiles : num_sms();
  rc = dispatch<kGateUp>(act_dtype, scale_dtype, a, grid, smem, pdl, st);
  if (rc) return rc;

  GemvParams d = {};
  d.packed = dn_packed; d.scale = dn_scale; d.zeros = dn_zeros;
  d.E = E; d.R = H; d.Rs = H; d.K = I; d.group = group;
  d.x = act; d.x_col_stride = I; d.x_slot_stride = (long long)kMaxTokens * I; d.ncols = T;
  d.plan = plan; d.I = I;
  d.out = out; d.out_col_stride = H;
  d.residual = residual; d.res_col_stride = H;
  d.err = err;
  d.prefetch = pdl ? 1 : 0;
  d.x_per_stage = 1;
  smem = plan_geometry(d, dn_zeros != nullptr, kDefaultSmemBudget);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  tiles = (H + 15) / 16;
  grid = tiles < num_sms() ? tiles : num_sms();
  return dispatch<kDown>(act_dtype, scale_dtype, d, grid, smem, pdl, st);
}

}  // namespace duplex
