// int4 dequant-GEMV family for batch <= 8 on sm_100a, over tile records (tiles.cuh).
//
// One persistent CTA per SM = 8 consumer warps + 1 producer warp.
//
// Producer (one lane): a stage is one tile record (16 weight rows x all K, with
// their scales and zero points) or two adjacent records (gate block + up block),
// fetched with ONE 1-D bulk copy (cp.async.bulk, no multicast) into a ring of
// shared-memory stages; per-stage activations (down projection: one row per
// token) follow with one bulk copy per row.  Completion is mbarrier transaction
// bytes; stages are recycled through a second mbarrier per slot.
//
// Consumers: the work of a stage is split into items = (record, 64-column pair);
// warp w takes items w, w+8, ...  Per item a lane does one 16-byte shared load of
// its weight words (rows g and g+8, two 32-column windows), two 16-byte loads of
// activation fragments, turns the nibbles into exact 16-bit (n - z) values in
// registers (Dq<T>) and issues four m16n8k16 MMAs (the 8 batch rows are the N
// dimension), alternating two accumulator chains.  Group scales (and, in the MoE
// down projection, the per-token routing weights) are applied in fp32 per item.
// Warps' partial sums meet in shared memory once per output tile.
//
// Modes:
//   kPlain  : out[j][r] fp32 = W[sel[j]] . x_j                    (dequant_gemv)
//   kLinear : y[b][r] = round(round(W . x_b) + bias) (+ residual)    (TritonPackedLinear)
//   kGateUp : unit u, row block j: act = silu(gate) * up, written in fragment order
//   kDown   : row block j over all units, routing-weighted combine (+ residual)
//
// PDL: kLinear / kDown issue their weight copies before griddepcontrol.wait;
// kDown also reads the routing plan there, because the gate|up kernel triggers
// its dependents only after its own wait on the router has returned.
#include "common.cuh"
#include "moe.cuh"
#include "tiles.cuh"
#include "gemv_core.cuh"

#include <mutex>
#include <set>
#include <utility>

namespace duplex {

constexpr int kStagesMax = 16;

enum : int { kPlain = 0, kLinear = 1, kGateUp = 2, kDown = 3 };
enum : int { kXShared = 0, kXStageFrag = 1, kXStageRaw = 2 };

// fixed shared-memory map (bytes)
constexpr uint32_t kOffFull = 0;       // kStagesMax mbarriers
constexpr uint32_t kOffEmpty = 128;    // kStagesMax mbarriers
constexpr uint32_t kOffAbort = 256;    // int
constexpr uint32_t kOffNUnits = 260;   // int
constexpr uint32_t kOffXslot = 320;    // kStagesMax ints (producer bookkeeping)
constexpr uint32_t kOffUnitE = 384;    // kMaxUnits ints
constexpr uint32_t kOffUnitM = 640;    // kMaxUnits uints
constexpr uint32_t kOffUnitW = 1024;   // kMaxUnits * kMaxTokens floats
constexpr uint32_t kOffRed = 3072;     // kCW * 8 * 32 floats
constexpr uint32_t kOffCorr = kOffRed + kCW * 8 * 32 * 4;  // npairs x 32 correction words

struct GemvParams {
  const uint8_t* tiles;
  int E, R, Rb;          // rows used, records per expert
  TileGeom tg;
  const void* x;
  long long x_col_stride;   // elements between batch columns
  long long x_slot_stride;  // elements between slots / units (per-stage activations)
  int ncols;
  int x_mode;
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
  int nstages, nrec;
  uint32_t stage_bytes, off_x, x_pitch, xbytes_row, smem_stage0, off_xsh;
  int prefetch;
  float rms_eps;
};

template <int MODE>
DEVI int tiles_of(const GemvParams& p, int n_units) {
  if (MODE == kPlain) return p.nslots * p.Rb;
  if (MODE == kLinear) return p.Rb;
  if (MODE == kGateUp) return n_units * (p.Rb >> 1);
  return p.Rb;  // kDown
}

template <int MODE>
DEVI int stages_of(int n_units) {
  return MODE == kDown ? n_units : 1;
}

// stage -> (expert, first record of the copy, activation slot)
template <int MODE>
DEVI void stage_decode(const GemvParams& p, const int* unit_e, int tile, int s, int& expert,
                       int& rec, int& xs) {
  if (MODE == kPlain) {
    const int slot = tile / p.Rb;
    rec = tile - slot * p.Rb;
    expert = p.sel[slot];
    xs = slot;
  } else if (MODE == kLinear) {
    expert = 0;
    rec = tile;
    xs = 0;
  } else if (MODE == kGateUp) {
    const int per = p.Rb >> 1;
    const int u = tile / per;
    rec = 2 * (tile - u * per);
    expert = unit_e[u];
    xs = u;
  } else {
    rec = tile;
    expert = unit_e[s];
    xs = s;
  }
}

template <typename T, typename S, int MODE, bool G32, bool CORR>
__global__ void __launch_bounds__(kThreads, 1) dq_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  int* n_units_s = reinterpret_cast<int*>(smem + kOffNUnits);
  int* xslot_of = reinterpret_cast<int*>(smem + kOffXslot);
  int* unit_e = reinterpret_cast<int*>(smem + kOffUnitE);
  uint32_t* unit_m = reinterpret_cast<uint32_t*>(smem + kOffUnitM);
  float* unit_w = reinterpret_cast<float*>(smem + kOffUnitW);

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

  if (warp == kCW) {
    // ------------------------------------------------------------ producer warp
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
      for (int u = lane; u < n_units; u += 32) unit_e[u] = p.plan->unit_expert[u];
      if (lane == 0) *n_units_s = n_units;
      __syncwarp();
    }
    const int ntiles = tiles_of<MODE>(p, n_units);
    const int nst = stages_of<MODE>(n_units);
    const uint32_t wbytes = (uint32_t)p.nrec * p.tg.rec_bytes;
    const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(p.x);

    auto issue_x = [&](int j) {
      const int slot = j % NS;
      if (p.x_mode != kXShared) {
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
        int expert, rec, xs;
        stage_decode<MODE>(p, unit_e, tile, s, expert, rec, xs);
        if ((unsigned)expert >= (unsigned)p.E) {
          if (lane == 0) set_error(p.err, DUPLEX_DEVERR_EXPERT);
          expert = 0;
        }
        if (lane == 0) {
          xslot_of[slot] = xs;
          mbar_arrive_expect_tx(&full[slot], wbytes);
          const uint8_t* src =
              p.tiles + ((size_t)expert * (size_t)p.Rb + (size_t)rec) * (size_t)p.tg.rec_bytes;
          bulk_g2s_stream(smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes, src, wbytes,
                          &full[slot], pol);
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
  uint8_t* xsh = smem + p.off_xsh;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  uint32_t* corr = reinterpret_cast<uint32_t*>(smem + kOffCorr);
  const TileGeom& tg = p.tg;

  int n_units = 0;
  if (MODE == kGateUp || MODE == kDown) {
    n_units = p.plan->n_units;
    n_units = n_units < 0 ? 0 : (n_units > kMaxUnits ? kMaxUnits : n_units);
    for (int u = tid; u < n_units; u += kConsumers) unit_m[u] = p.plan->unit_mask[u];
    if (MODE == kDown)
      for (int idx = tid; idx < n_units * kMaxTokens; idx += kConsumers)
        unit_w[idx] = p.plan->unit_w[idx];
  }
  if (p.x_mode == kXShared) {
    stage_x_shared<T, CORR>(xsh, p.x_pitch, reinterpret_cast<const uint8_t*>(p.x), p.x_col_stride,
                            p.ncols, tg, p.rms_eps, red, tid, warp, lane);
    if (CORR) build_corr<T>(corr, xsh, p.x_pitch, tg.npairs, p.ncols, tid);
  }
  named_bar_sync(1, kConsumers);
  // zero the padded activation tail of every per-stage activation row (never copied)
  if (p.x_mode != kXShared && tg.Kp > tg.K) {
    const int tail = (tg.Kp - tg.K) * 2;
    for (int s = 0; s < NS; ++s)
      for (int idx = tid; idx < p.ncols * tail; idx += kConsumers) {
        const int n = idx / tail, b = idx - n * tail;
        smem[p.smem_stage0 + (uint32_t)s * p.stage_bytes + p.off_x + (uint32_t)n * p.x_pitch +
             (uint32_t)tg.K * 2u + b] = 0;
      }
    named_bar_sync(1, kConsumers);
  }

  const int ntiles = tiles_of<MODE>(p, n_units);
  const int nst = stages_of<MODE>(n_units);
  const bool xon = g < p.ncols;
  const bool xraw = p.x_mode == kXStageRaw;
  const int npairs = tg.npairs;
  const int ips = p.nrec * npairs;  // items per stage

  if (MODE == kLinear && CORR && ntiles > (int)gridDim.x) {
    // Dense linear with more tiles than CTAs (q, fused q|k|v, lm_head; a tile is one
    // stage): each warp's partial sums of
    // up to `rmax` tiles wait in `red` ([tile][warp][column][row]); one consumer barrier
    // and one pass then reduce them (warps in order) and write the rows.  The ring
    // position advances stage by stage.
    const int per = p.ncols * 16;
    int rmax = (kCW * 8 * 32) / (kCW * per);
    if (rmax > kConsumers / per) rmax = kConsumers / per;
    const int lo = (warp * ips) / kCW, hi = ((warp + 1) * ips) / kCW;
    int slot = 0;
    uint32_t phase = 0u;
    int j = 0, t0 = blockIdx.x;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      if (!mbar_wait_bounded(&full[slot], phase, abort_flag)) {
        if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
      }
      const uint8_t* st = smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f};
      float acc1[4] = {0.f, 0.f, 0.f, 0.f};
      consume_corr<T, S, G32>(st, tg, lo, hi, lane, xsh, p.x_pitch, corr, xon, acc0, acc1);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == NS) {
        slot = 0;
        phase ^= 1u;
      }
      float* b = red + (j * kCW + warp) * per;
      if (2 * t < p.ncols) {
        b[(2 * t) * 16 + g] = acc0[0];
        b[(2 * t) * 16 + g + 8] = acc0[2];
      }
      if (2 * t + 1 < p.ncols) {
        b[(2 * t + 1) * 16 + g] = acc0[1];
        b[(2 * t + 1) * 16 + g + 8] = acc0[3];
      }
      if (++j == rmax || tile + (int)gridDim.x >= ntiles) {
        named_bar_sync(1, kConsumers);
        for (int o = tid; o < j * per; o += kConsumers) {
          const int jj = o / per, rem = o - jj * per;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kCW; ++w) v += red[(jj * kCW + w) * per + rem];
          const int n = rem >> 4, row = (t0 + jj * (int)gridDim.x) * 16 + (rem & 15);
          if (row < p.R) {
            T y = from_f32<T>(v);
            if (p.bias)
              y = from_f32<T>(to_f32<T>(y) + to_f32<T>(reinterpret_cast<const T*>(p.bias)[row]));
            if (p.residual)
              y = from_f32<T>(to_f32<T>(y) + to_f32<T>(reinterpret_cast<const T*>(
                                                  p.residual)[n * p.res_col_stride + row]));
            reinterpret_cast<T*>(p.out)[n * p.out_col_stride + row] = y;
          }
        }
        named_bar_sync(1, kConsumers);
        j = 0;
        t0 = tile + (int)gridDim.x;
      }
    }
    return;
  }

  int i = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float acc0[4] = {0.f, 0.f, 0.f, 0.f};
    float acc1[4] = {0.f, 0.f, 0.f, 0.f};
    const int npt = nst * ips;
    const int ib = (warp * npt) / kCW, ie = ((warp + 1) * npt) / kCW;

    for (int s = 0; s < nst; ++s, ++i) {
      const int slot = i % NS;
      if (!mbar_wait_bounded(&full[slot], (uint32_t)(i / NS) & 1u, abort_flag)) {
        if (lane == 0) set_error(p.err, DUPLEX_DEVERR_TIMEOUT);
      }
      const uint8_t* st = smem + p.smem_stage0 + (uint32_t)slot * p.stage_bytes;
      const int lo = ib > s * ips ? ib - s * ips : 0;
      const int hi = ie < (s + 1) * ips ? ie - s * ips : ips;
      if (CORR) {
        consume_corr<T, S, G32>(st, tg, lo, hi, lane, xsh, p.x_pitch, corr, xon, acc0, acc1);
      } else {
        const uint8_t* xrow = st + p.off_x + (uint32_t)g * p.x_pitch + (uint32_t)t * 16u;
        float w0 = 1.f, w1 = 1.f;
        if (MODE == kDown) {
          w0 = unit_w[s * kMaxTokens + 2 * t];
          w1 = unit_w[s * kMaxTokens + 2 * t + 1];
        }
#pragma unroll 2
        for (int it = lo; it < hi; ++it)
          item_exact<T, S, G32>(st, tg, it, lane, xrow, xon, xraw, w0, w1, acc0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---- split-K reduction across the consumer warps, then the epilogue
    float v, v2;
    reduce_tile(red, acc0, acc1, MODE == kGateUp, tid, warp, lane, v, v2);
    if (tid < 128) {
      const int n = tid >> 4, r = tid & 15;
      if (MODE == kPlain) {
        const int slot = tile / p.Rb;
        const int row = (tile - slot * p.Rb) * 16 + r;
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
        const int per = p.Rb >> 1;
        const int u = tile / per;
        const int row = (tile - u * per) * 16 + r;
        if (n < p.ncols) {
          const float a = ((unit_m[u] >> n) & 1u) ? silu_f32(v) * v2 : 0.f;
          reinterpret_cast<T*>(p.out)[((size_t)u * kMaxTokens + n) * p.I + frag_pos(row)] =
              from_f32<T>(a);
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

// ---------------------------------------------------------------------- repack
template <typename S>
__global__ void repack_kernel(const int32_t* __restrict__ packed, const S* __restrict__ scale,
                              const int32_t* __restrict__ zeros, int E, int R, int Rb, int C, int G,
                              int GZ, TileGeom tg, int pair_halves, uint32_t* __restrict__ tiles) {
  const uint32_t wpr = tg.rec_bytes / 4u;
  const long long total = (long long)E * Rb * wpr;
  const int half = Rb >> 1;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long recg = idx / wpr;
    const uint32_t o = (uint32_t)(idx - recg * wpr) * 4u;
    const int e = (int)(recg / Rb);
    const int rout = (int)(recg - (long long)e * Rb);
    const int rb = pair_halves ? ((rout & 1) ? half + (rout >> 1) : (rout >> 1)) : rout;
    uint32_t val = 0;
    if (o < tg.off_scale) {
      const int pr = (int)(o >> 9);
      const int ln = (int)((o & 511u) >> 4);
      const int j = (int)((o & 15u) >> 2);
      const int g = ln >> 2, t = ln & 3;
      const int row = rb * 16 + g + ((j & 1) ? 8 : 0);
      const int word = 8 * pr + t + ((j & 2) ? 4 : 0);
      if (row < R && word < C) val = (uint32_t)packed[((long long)e * R + row) * C + word];
    } else if (o < tg.off_zero) {
      const int q = (int)((o - tg.off_scale) >> 2);
      const int grp = q >> 3, g = q & 7;
      const int ra = rb * 16 + g, rbw = ra + 8;
      uint16_t sa = 0, sb = 0;
      if (grp < G) {
        if (ra < R) sa = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * R + ra) * G + grp]);
        if (rbw < R) sb = *reinterpret_cast<const uint16_t*>(&scale[((long long)e * R + rbw) * G + grp]);
      }
      val = (uint32_t)sa | ((uint32_t)sb << 16);
    } else if (tg.has_zeros && o < tg.off_zero + (uint32_t)tg.Gr * 8u) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int q = (int)(o - tg.off_zero) + b;
        const int grp = q >> 3, g = q & 7;
        const int ra = rb * 16 + g, rbw = ra + 8;
        uint32_t za = 0, zb = 0;
        if (grp < G) {
          if (ra < R)
            za = ((uint32_t)zeros[((long long)e * R + ra) * GZ + (grp >> 3)] >> ((grp & 7) * 4)) & 15u;
          if (rbw < R)
            zb = ((uint32_t)zeros[((long long)e * R + rbw) * GZ + (grp >> 3)] >> ((grp & 7) * 4)) & 15u;
        }
        val |= (za | (zb << 4)) << (8 * b);
      }
    }
    tiles[idx] = val;
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

constexpr size_t kMaxSmem = 227 * 1024;
size_t g_smem_linear = 112 * 1024, g_smem_gateup = 148 * 1024, g_smem_down = 76 * 1024,
       g_smem_plain = 112 * 1024;

// Fill the shared-memory geometry of `p`; returns the dynamic smem bytes or 0.
static size_t plan_geometry(GemvParams& p, size_t budget) {
  p.x_pitch = up((uint32_t)p.tg.Kp * 2u, 128) + 64u;
  p.xbytes_row = (uint32_t)p.tg.K * 2u;
  p.off_x = (uint32_t)p.nrec * p.tg.rec_bytes;
  const uint32_t sb = p.off_x + (p.x_mode != kXShared ? (uint32_t)p.ncols * p.x_pitch : 0u);
  p.stage_bytes = up(sb, 128);
  const uint32_t corr_bytes = p.x_mode == kXShared ? (uint32_t)p.tg.npairs * 128u : 0u;
  p.off_xsh = up(kOffCorr + corr_bytes, 128);
  p.smem_stage0 = up(p.off_xsh + (p.x_mode == kXShared ? (uint32_t)p.ncols * p.x_pitch : 0u), 128);
  size_t b = budget < kMaxSmem ? budget : kMaxSmem;
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

// cudaFuncAttributeMaxDynamicSharedMemorySize, once per (kernel, device)
int ensure_smem_attr(const void* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return DUPLEX_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return record_cuda(e);
  done.insert({fn, dev});
  return DUPLEX_OK;
}

template <typename T, typename S, int MODE, bool G32>
static int launch(GemvParams& p, int grid, size_t smem, bool pdl, cudaStream_t stream) {
  // offset dequant + correction MMA wherever the activations are shared by all stages
  const bool corr = p.x_mode == kXShared;
  void (*kern)(GemvParams) = corr ? dq_gemv_kernel<T, S, MODE, G32, true>
                                  : dq_gemv_kernel<T, S, MODE, G32, false>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kMaxSmem);
  if (rc) return rc;
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

template <int MODE, bool G32>
static int dispatch_g(int act_dtype, int scale_dtype, GemvParams& p, int grid, size_t smem, bool pdl,
                      cudaStream_t st) {
  if (act_dtype == DUPLEX_DTYPE_F16 && scale_dtype == DUPLEX_DTYPE_F16)
    return launch<__half, __half, MODE, G32>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_F16 && scale_dtype == DUPLEX_DTYPE_BF16)
    return launch<__half, __nv_bfloat16, MODE, G32>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_BF16 && scale_dtype == DUPLEX_DTYPE_BF16)
    return launch<__nv_bfloat16, __nv_bfloat16, MODE, G32>(p, grid, smem, pdl, st);
  if (act_dtype == DUPLEX_DTYPE_BF16 && scale_dtype == DUPLEX_DTYPE_F16)
    return launch<__nv_bfloat16, __half, MODE, G32>(p, grid, smem, pdl, st);
  return DUPLEX_ERR_DTYPE;
}

template <int MODE>
static int dispatch(int act_dtype, int scale_dtype, GemvParams& p, int grid, size_t smem, bool pdl,
                    cudaStream_t st) {
  if (p.tg.gshift < 0) return dispatch_g<MODE, true>(act_dtype, scale_dtype, p, grid, smem, pdl, st);
  return dispatch_g<MODE, false>(act_dtype, scale_dtype, p, grid, smem, pdl, st);
}

static inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int check_tiles(const void* tiles, int scale_dtype, int E, int R, int K, int group,
                       int has_zeros, TileGeom* tg) {
  if (!tiles) return DUPLEX_ERR_ARG;
  if (E < 1 || R < 1 || K < 1 || group < 1) return DUPLEX_ERR_ARG;
  if (scale_dtype != DUPLEX_DTYPE_F16 && scale_dtype != DUPLEX_DTYPE_BF16) return DUPLEX_ERR_DTYPE;
  if (tile_geom(K, group, has_zeros, tg)) return DUPLEX_ERR_UNSUPPORTED;
  if (!al16(tiles)) return DUPLEX_ERR_ALIGN;
  return DUPLEX_OK;
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_tile_record_bytes(int32_t K, int32_t group, int has_zeros, size_t* bytes) {
  TileGeom tg;
  if (!bytes) return DUPLEX_ERR_ARG;
  if (tile_geom(K, group, has_zeros, &tg)) return DUPLEX_ERR_UNSUPPORTED;
  *bytes = tg.rec_bytes;
  return DUPLEX_OK;
}

extern "C" int duplex_repack_tiles(const int32_t* packed, const void* scale, const int32_t* zeros,
                                   int scale_dtype, int32_t E, int32_t R, int32_t K, int32_t group,
                                   int32_t pair_halves, void* tiles, size_t tiles_bytes,
                                   void* stream) {
  if (!packed || !scale || !tiles || E < 1 || R < 1) return DUPLEX_ERR_ARG;
  TileGeom tg;
  if (tile_geom(K, group, zeros != nullptr, &tg)) return DUPLEX_ERR_UNSUPPORTED;
  int Rb = (R + 15) / 16;
  if (pair_halves) {
    if ((R & 31) != 0) return DUPLEX_ERR_UNSUPPORTED;  // both halves whole 16-row blocks
  }
  if ((size_t)E * Rb * tg.rec_bytes > tiles_bytes) return DUPLEX_ERR_WORKSPACE;
  if (!al16(tiles)) return DUPLEX_ERR_ALIGN;
  const int C = K / 8, G = (K + group - 1) / group, GZ = (G + 7) / 8;
  const long long words = (long long)E * Rb * (tg.rec_bytes / 4);
  int blocks = (int)((words + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  cudaStream_t st = (cudaStream_t)stream;
  if (scale_dtype == DUPLEX_DTYPE_F16)
    repack_kernel<__half><<<blocks, 256, 0, st>>>(packed, reinterpret_cast<const __half*>(scale),
                                                   zeros, E, R, Rb, C, G, GZ, tg, pair_halves,
                                                   reinterpret_cast<uint32_t*>(tiles));
  else if (scale_dtype == DUPLEX_DTYPE_BF16)
    repack_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        packed, reinterpret_cast<const __nv_bfloat16*>(scale), zeros, E, R, Rb, C, G, GZ, tg,
        pair_halves, reinterpret_cast<uint32_t*>(tiles));
  else
    return DUPLEX_ERR_DTYPE;
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_dq_gemv(const void* x, int act_dtype, int64_t x_slot_stride, const void* tiles,
                              int scale_dtype, int has_zeros, int32_t E, int32_t R, int32_t K,
                              int32_t group, const int32_t* sel, int32_t nsel, float* out,
                              int32_t* err, void* stream) {
  GemvParams p = {};
  int rc = check_tiles(tiles, scale_dtype, E, R, K, group, has_zeros, &p.tg);
  if (rc) return rc;
  if (!x || !sel || !out || nsel < 1) return DUPLEX_ERR_ARG;
  if (!al16(x) || (x_slot_stride & 7)) return DUPLEX_ERR_ALIGN;
  p.tiles = reinterpret_cast<const uint8_t*>(tiles);
  p.E = E; p.R = R; p.Rb = (R + 15) / 16;
  p.x = x; p.x_col_stride = 0; p.x_slot_stride = x_slot_stride; p.ncols = 1;
  p.x_mode = x_slot_stride != 0 ? kXStageRaw : kXShared;
  p.sel = sel; p.nslots = nsel;
  p.out = out; p.out_slot_stride = R; p.out_col_stride = 0;
  p.err = err;
  p.nrec = 1;
  const size_t smem = plan_geometry(p, g_smem_plain);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  const int tiles_n = nsel * p.Rb;
  const int grid = tiles_n < num_sms() ? tiles_n : num_sms();
  return dispatch<kPlain>(act_dtype, scale_dtype, p, grid, smem, false, (cudaStream_t)stream);
}

extern "C" int duplex_packed_linear(const void* x, int act_dtype, int32_t B, int64_t x_row_stride,
                                    const void* tiles, int scale_dtype, int has_zeros, int32_t R,
                                    int32_t K, int32_t group, const void* bias,
                                    const void* residual, int64_t res_row_stride, void* out,
                                    int64_t out_row_stride, float rms_eps, int pdl, void* stream) {
  GemvParams p = {};
  int rc = check_tiles(tiles, scale_dtype, 1, R, K, group, has_zeros, &p.tg);
  if (rc) return rc;
  if (!x || !out || B < 1 || B > kMaxTokens) return DUPLEX_ERR_ARG;
  if (!al16(x) || (x_row_stride & 7)) return DUPLEX_ERR_ALIGN;
  p.tiles = reinterpret_cast<const uint8_t*>(tiles);
  p.E = 1; p.R = R; p.Rb = (R + 15) / 16;
  p.x = x; p.x_col_stride = x_row_stride; p.x_slot_stride = 0; p.ncols = B;
  p.x_mode = kXShared;
  p.out = out; p.out_slot_stride = 0; p.out_col_stride = out_row_stride;
  p.bias = bias; p.residual = residual; p.res_col_stride = res_row_stride;
  p.prefetch = pdl ? 1 : 0;
  p.rms_eps = rms_eps;
  p.nrec = 1;
  const size_t smem = plan_geometry(p, g_smem_linear);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  const int grid = p.Rb < num_sms() ? p.Rb : num_sms();
  return dispatch<kLinear>(act_dtype, scale_dtype, p, grid, smem, pdl != 0, (cudaStream_t)stream);
}

namespace duplex {

// Gate|up and down launches of the decode MoE (T <= 8); called by moe.cu.
int launch_moe_experts(int act_dtype, int scale_dtype, int has_zeros, int T, int E, int H, int I,
                       int group, const void* gu_tiles, const void* dn_tiles, const MoePlan* plan,
                       const void* x, void* act, const void* residual, void* out, int* err,
                       int max_units, bool pdl, cudaStream_t st) {
  GemvParams a = {};
  int rc = check_tiles(gu_tiles, scale_dtype, E, 2 * I, H, group, has_zeros, &a.tg);
  if (rc) return rc;
  GemvParams d = {};
  rc = check_tiles(dn_tiles, scale_dtype, E, H, I, group, has_zeros, &d.tg);
  if (rc) return rc;
  if ((I & 15) || (H & 7)) return DUPLEX_ERR_UNSUPPORTED;

  a.tiles = reinterpret_cast<const uint8_t*>(gu_tiles);
  a.E = E; a.R = 2 * I; a.Rb = 2 * I / 16;
  a.x = x; a.x_col_stride = H; a.x_slot_stride = 0; a.ncols = T;
  a.x_mode = kXShared;
  a.plan = plan; a.I = I;
  a.out = act;
  a.err = err;
  a.prefetch = 0;
  a.nrec = 2;
  size_t smem = plan_geometry(a, g_smem_gateup);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  int tiles_n = max_units * (I / 16);
  int grid = tiles_n < num_sms() ? tiles_n : num_sms();
  rc = dispatch<kGateUp>(act_dtype, scale_dtype, a, grid, smem, pdl, st);
  if (rc) return rc;

  d.tiles = reinterpret_cast<const uint8_t*>(dn_tiles);
  d.E = E; d.R = H; d.Rb = (H + 15) / 16;
  d.x = act; d.x_col_stride = I; d.x_slot_stride = (long long)kMaxTokens * I; d.ncols = T;
  d.x_mode = kXStageFrag;
  d.plan = plan; d.I = I;
  d.out = out; d.out_col_stride = H;
  d.residual = residual; d.res_col_stride = H;
  d.err = err;
  d.prefetch = pdl ? 1 : 0;
  d.nrec = 1;
  smem = plan_geometry(d, g_smem_down);
  if (!smem) return DUPLEX_ERR_UNSUPPORTED;
  tiles_n = d.Rb;
  grid = tiles_n < num_sms() ? tiles_n : num_sms();
  return dispatch<kDown>(act_dtype, scale_dtype, d, grid, smem, pdl, st);
}

}  // namespace duplex
