// Consumer-side building blocks of the int4 dequant-GEMV kernels (gemv.cu and the
// persistent clock-path kernel in stack.cu): activation staging in MMA fragment
// order, the exact and the offset dequantisation paths, and the per-pair
// correction table.  All of them assume 16 consumer warps (named barrier 1).
#pragma once

#include "common.cuh"
#include "tiles.cuh"

namespace duplex {

constexpr int kCW = 16;  // consumer warps
constexpr int kConsumers = kCW * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp

DEVI bool wait_limited(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// position of logical column c inside its 8-column group in fragment order
// (stored sequence x0 x4 x1 x5 x2 x6 x3 x7)
DEVI int frag_pos(int c) {
  const int r = c & 7;
  return (c & ~7) | ((r & 3) << 1) | (r >> 2);
}

DEVI uint4 to_frag_order(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
  o.y = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
  o.z = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
  o.w = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
  return o;
}

DEVI float2 scale_pair(uint32_t s2, __half*) { return __half22float2(*reinterpret_cast<__half2*>(&s2)); }
DEVI float2 scale_pair(uint32_t s2, __nv_bfloat16*) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&s2));
}

// ---- exact path (per-stage activations): item = (record, column pair p)
// acc += (scale * colw) * sum over the pair of (n - z) * x
template <typename T, typename S, bool G32>
DEVI void item_exact(const uint8_t* rec, const TileGeom& tg, int p, int lane, const uint8_t* xrow,
                     bool xon, bool xraw, float w0, float w1, float (&acc)[4]) {
  const int g = lane >> 2;
  const uint4 w = *reinterpret_cast<const uint4*>(rec + (((uint32_t)p << 5) + lane) * 16u);
  uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
  if (xon) {
    xa = *reinterpret_cast<const uint4*>(xrow + (uint32_t)p * 128u);
    xb = *reinterpret_cast<const uint4*>(xrow + (uint32_t)p * 128u + 64u);
    if (xraw) {
      xa = to_frag_order(xa);
      xb = to_frag_order(xb);
    }
  }
  const uint32_t* sc = reinterpret_cast<const uint32_t*>(rec + tg.off_scale);
  const uint8_t* zr = rec + tg.off_zero;
  uint32_t A[4], B[4], lo_a, hi_a, lo_b, hi_b;
#pragma unroll
  for (int h = 0; h < (G32 ? 2 : 1); ++h) {
    const int grp = G32 ? 2 * p + h : (p >> tg.gshift);
    const uint32_t zz = tg.has_zeros ? (uint32_t)zr[grp * 8 + g] : 0x88u;
    Dq<T>::consts(zz & 15u, lo_a, hi_a);
    Dq<T>::consts(zz >> 4, lo_b, hi_b);
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    if (!G32 || h == 0) {
      Dq<T>::expand(w.x, w.y, lo_a, hi_a, lo_b, hi_b, A, B);
      MmaOp<T>::run(c0, A[0], A[1], A[2], A[3], xa.x, xa.y);
      MmaOp<T>::run(c1, B[0], B[1], B[2], B[3], xa.z, xa.w);
    }
    if (!G32 || h == 1) {
      Dq<T>::expand(w.z, w.w, lo_a, hi_a, lo_b, hi_b, A, B);
      MmaOp<T>::run(c0, A[0], A[1], A[2], A[3], xb.x, xb.y);
      MmaOp<T>::run(c1, B[0], B[1], B[2], B[3], xb.z, xb.w);
    }
    const float2 s = scale_pair(sc[grp * 8 + g], (S*)nullptr);
    acc[0] = fmaf(s.x * w0, c0[0] + c1[0], acc[0]);
    acc[1] = fmaf(s.x * w1, c0[1] + c1[1], acc[1]);
    acc[2] = fmaf(s.y * w0, c0[2] + c1[2], acc[2]);
    acc[3] = fmaf(s.y * w1, c0[3] + c1[3], acc[3]);
  }
}

// ---- offset path (shared activations): per column pair, four MMAs of (M + n) x
// plus one correction MMA (corr_a coefficients x the pair's exact column sums);
// the group scale is applied when the warp's run of a group ends.
template <typename T, typename S>
struct OffAcc {
  float d0[4], d1[4];
  int rec, grp;
  uint32_t ca0, ca1;
  DEVI void reset() {
#pragma unroll
    for (int r = 0; r < 4; ++r) d0[r] = d1[r] = 0.f;
  }
  DEVI void window(uint32_t wa, uint32_t wb, uint4 xv) {
    uint32_t A[4], B[4];
    DqOff<T>::expand(wa, wb, A, B);
    MmaOp<T>::run(d0, A[0], A[1], A[2], A[3], xv.x, xv.y);
    MmaOp<T>::run(d1, B[0], B[1], B[2], B[3], xv.z, xv.w);
  }
  DEVI void set_group(const uint8_t* r, const TileGeom& tg, int lane, uint32_t wmask) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t zz = tg.has_zeros ? (uint32_t)r[tg.off_zero + grp * 8 + g] : 0x88u;
    DqOff<T>::corr_a(zz & 15u, zz >> 4, t, wmask, ca0, ca1);
  }
  DEVI void correct(uint32_t bcorr) { MmaOp<T>::run(d0, ca0, ca1, 0u, 0u, bcorr, 0u); }
  DEVI void flush(const uint8_t* r, const TileGeom& tg, int lane, float (&acc)[4]) {
    const int g = lane >> 2;
    const float2 s = scale_pair(reinterpret_cast<const uint32_t*>(r + tg.off_scale)[grp * 8 + g],
                                (S*)nullptr);
    acc[0] = fmaf(s.x, d0[0] + d1[0], acc[0]);
    acc[1] = fmaf(s.x, d0[1] + d1[1], acc[1]);
    acc[2] = fmaf(s.y, d0[2] + d1[2], acc[2]);
    acc[3] = fmaf(s.y, d0[3] + d1[3], acc[3]);
  }
};


// Stage ncols activation rows of K (global, rows `col_stride` elements apart) into
// shared memory in fragment order, zero-padded to Kp; with `rms_eps > 0` each row is
// RMS-normalised first (weightless RMSNorm, rounded to T).  With the offset path
// (CORR, fp16) odd columns are stored divided by 16.  `red` provides 16 x 8 + 8
// floats of scratch.  `plain`, when given, also receives the (normalised) rows in
// natural order, [ncols][K].  Ends with a consumer-wide barrier.  Activations are
// read through L2 (ld.global.cg): other CTAs may have written them.
template <typename T, bool CORR>
DEVI void stage_x_shared(uint8_t* xsh, uint32_t pitch, const uint8_t* xb, long long col_stride,
                         int ncols, const TileGeom& tg, float rms_eps, float* red, int tid, int warp,
                         int lane, uint8_t* plain = nullptr) {
  const int nq = tg.Kp >> 3;
  float* invs = red + kCW * 8;  // per-row RMS scale
  if (rms_eps > 0.f) {
    for (int n = 0; n < ncols; ++n) {
      float a = 0.f;
      for (int q = tid; q < (tg.K >> 3); q += kConsumers) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xb + ((size_t)n * col_stride + q * 8) * 2));
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) a = fmaf(to_f32<T>(e[k]), to_f32<T>(e[k]), a);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) red[warp * 8 + n] = a;
    }
    named_bar_sync(1, kConsumers);
    if (tid < ncols) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) tot += red[w * 8 + tid];
      invs[tid] = 1.0f / sqrtf(tot / (float)tg.K + rms_eps);
    }
    named_bar_sync(1, kConsumers);
  }
  for (int idx = tid; idx < ncols * nq; idx += kConsumers) {
    const int n = idx / nq, q = idx - n * nq;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q * 8 < tg.K) {
      v = __ldcg(reinterpret_cast<const uint4*>(xb + ((size_t)n * col_stride + q * 8) * 2));
      if (rms_eps > 0.f) {
        const float inv = invs[n];
        T* e = reinterpret_cast<T*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = from_f32<T>(to_f32<T>(e[k]) * inv);
      }
    }
    if (plain && q * 8 < tg.K)
      *reinterpret_cast<uint4*>(plain + ((size_t)n * tg.K + q * 8) * 2) = v;
    uint4 o = to_frag_order(v);
    if (CORR && DqOff<T>::kOddDiv16) {
      const __half2 q16 = __float2half2_rn(0.0625f);
      __half2 hy = __hmul2(*reinterpret_cast<__half2*>(&o.y), q16);
      __half2 hw = __hmul2(*reinterpret_cast<__half2*>(&o.w), q16);
      o.y = *reinterpret_cast<uint32_t*>(&hy);
      o.w = *reinterpret_cast<uint32_t*>(&hw);
    }
    *reinterpret_cast<uint4*>(xsh + (uint32_t)n * pitch + (uint32_t)q * 16u) = o;
  }
  named_bar_sync(1, kConsumers);
}

// Correction table of the offset path: word (pair p, lane g*4 + t) is the B
// fragment of the pair's correction MMA for column g -- exact activation sums of
// the pair's 32-column windows in 16-bit parts (t = 0 / 1: window 2p, t = 2 / 3:
// window 2p + 1; fp16 splits even / odd columns, bf16 uses three parts).  Reads the
// staged (fragment-ordered) activations.  Caller synchronises before use.
template <typename T>
DEVI void build_corr(uint32_t* corr, const uint8_t* xsh, uint32_t pitch, int npairs, int ncols,
                     int tid) {
  for (int idx = tid; idx < npairs * 8; idx += kConsumers) {
    const int pp = idx >> 3, n = idx & 7;
    uint32_t b[4] = {0u, 0u, 0u, 0u};
    if (n < ncols) {
      const uint8_t* row = xsh + (uint32_t)n * pitch + (uint32_t)pp * 128u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float se = 0.f, so = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 o = *reinterpret_cast<const uint4*>(row + h * 64 + q * 16);
          const T* e = reinterpret_cast<const T*>(&o);
          // fragment order: e0 = x0, e1 = x4, e2 = x1, e3 = x5, e4 = x2, e5 = x6, e6 = x3, e7 = x7
          se += (to_f32<T>(e[0]) + to_f32<T>(e[1])) + (to_f32<T>(e[4]) + to_f32<T>(e[5]));
          so += (to_f32<T>(e[2]) + to_f32<T>(e[3])) + (to_f32<T>(e[6]) + to_f32<T>(e[7]));
        }
        if (DqOff<T>::kOddDiv16) {
          so *= 16.f;
          const T eh = from_f32<T>(se), oh = from_f32<T>(so);
          const T el = from_f32<T>(se - to_f32<T>(eh)), ol = from_f32<T>(so - to_f32<T>(oh));
          b[2 * h] = (uint32_t)*reinterpret_cast<const uint16_t*>(&eh) |
                     ((uint32_t)*reinterpret_cast<const uint16_t*>(&el) << 16);
          b[2 * h + 1] = (uint32_t)*reinterpret_cast<const uint16_t*>(&oh) |
                         ((uint32_t)*reinterpret_cast<const uint16_t*>(&ol) << 16);
        } else {
          const float x = se + so;
          const T x1 = from_f32<T>(x);
          const T x2 = from_f32<T>(x - to_f32<T>(x1));
          const T x3 = from_f32<T>(x - to_f32<T>(x1) - to_f32<T>(x2));
          b[2 * h] = (uint32_t)*reinterpret_cast<const uint16_t*>(&x1) |
                     ((uint32_t)*reinterpret_cast<const uint16_t*>(&x2) << 16);
          b[2 * h + 1] = (uint32_t)*reinterpret_cast<const uint16_t*>(&x3);
        }
      }
    }
    *reinterpret_cast<uint4*>(corr + pp * 32 + n * 4) = make_uint4(b[0], b[1], b[2], b[3]);
  }
}

// Offset-path items [lo, hi) of a stage holding `nrec` records (items [0, npairs)
// are record 0, [npairs, 2 npairs) record 1).  acc0 / acc1 collect records 0 / 1.
template <typename T, typename S, bool G32>
DEVI void consume_corr(const uint8_t* st, const TileGeom& tg, int lo, int hi, int lane,
                       const uint8_t* xsh, uint32_t pitch, const uint32_t* corr, bool xon,
                       float (&acc0)[4], float (&acc1)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const int npairs = tg.npairs;
  const uint8_t* xrow = xsh + (uint32_t)g * pitch + (uint32_t)t * 16u;
  OffAcc<T, S> oa;
  oa.reset();
  oa.rec = -1;
  oa.grp = -1;
  for (int it = lo; it < hi; ++it) {
    const int r = it >= npairs ? 1 : 0;
    const int pp = it - r * npairs;
    const uint8_t* rec = st + (uint32_t)r * tg.rec_bytes;
    const uint4 w = *reinterpret_cast<const uint4*>(rec + (((uint32_t)pp << 5) + lane) * 16u);
    const uint32_t bc = corr[pp * 32 + lane];
    uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
    if (xon) {
      xa = *reinterpret_cast<const uint4*>(xrow + (uint32_t)pp * 128u);
      xb = *reinterpret_cast<const uint4*>(xrow + (uint32_t)pp * 128u + 64u);
    }
    if (G32) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        oa.reset();
        oa.grp = 2 * pp + h;
        oa.set_group(rec, tg, lane, 1u << h);
        oa.window(h ? w.z : w.x, h ? w.w : w.y, h ? xb : xa);
        oa.correct(bc);
        oa.flush(rec, tg, lane, r ? acc1 : acc0);
      }
    } else {
      const int grp = pp >> tg.gshift;
      if (grp != oa.grp || r != oa.rec) {
        if (oa.grp >= 0)
          oa.flush(st + (uint32_t)oa.rec * tg.rec_bytes, tg, lane, oa.rec ? acc1 : acc0);
        oa.reset();
        oa.grp = grp;
        oa.rec = r;
        oa.set_group(rec, tg, lane, 3u);
      }
      oa.window(w.x, w.y, xa);
      oa.window(w.z, w.w, xb);
      oa.correct(bc);
    }
  }
  if (!G32 && oa.grp >= 0)
    oa.flush(st + (uint32_t)oa.rec * tg.rec_bytes, tg, lane, oa.rec ? acc1 : acc0);
}

// ---- offset path with the correction applied in fp32, once per group --------
// The MMAs of one group accumulate D = sum (M + n) x' over the group's columns,
// x' being the staged activations (fp16: odd columns stored / 16).  With the
// per-token sums of the columns covered
//   fp16: P = 1024 (SE + SO'),  Q = SE + 16 SO'   (SE: even columns, SO': odd, staged)
//   bf16: P = 128 SX,            Q = SX
// the exact dot product is D - P - z Q; it is scaled by the group scale (and a
// per-column weight) in fp32.  `gsum` holds (P, Q) as float2 [unit][8 tokens] per
// 64-column pair (per 32-column window when the group is 32), so a warp that
// covers only part of a group subtracts exactly the part it covered; lane (g, t)
// reads tokens 2t, 2t + 1 as one float4.
template <typename S>
DEVI void flush_group(float (&acc)[4], const float (&d0)[4], const float (&d1)[4],
                      const uint8_t* rec, const TileGeom& tg, int grp, int g, float4 gs,
                      float w0, float w1) {
  const uint32_t zz = tg.has_zeros ? (uint32_t)rec[tg.off_zero + grp * 8 + g] : 0x88u;
  const float za = (float)(zz & 15u), zb = (float)(zz >> 4);
  const float2 s =
      scale_pair(reinterpret_cast<const uint32_t*>(rec + tg.off_scale)[grp * 8 + g], (S*)nullptr);
  acc[0] = fmaf(s.x * w0, (d0[0] + d1[0]) - fmaf(za, gs.y, gs.x), acc[0]);
  acc[1] = fmaf(s.x * w1, (d0[1] + d1[1]) - fmaf(za, gs.w, gs.z), acc[1]);
  acc[2] = fmaf(s.y * w0, (d0[2] + d1[2]) - fmaf(zb, gs.y, gs.x), acc[2]);
  acc[3] = fmaf(s.y * w1, (d0[3] + d1[3]) - fmaf(zb, gs.w, gs.z), acc[3]);
}

template <typename T>
DEVI void mma_window(float (&d0)[4], float (&d1)[4], uint32_t wa, uint32_t wb, uint4 x) {
  uint32_t A[4], B[4];
  DqOff<T>::expand(wa, wb, A, B);
  MmaOp<T>::run(d0, A[0], A[1], A[2], A[3], x.x, x.y);
  MmaOp<T>::run(d1, B[0], B[1], B[2], B[3], x.z, x.w);
}

DEVI void zero4(float (&d)[4]) { d[0] = d[1] = d[2] = d[3] = 0.f; }

// Pair-major walk over column pairs [pb, pe) of the NREC records of a stage that
// share one set of staged activation rows (xsh, fragment order): each pair's
// activation fragments are loaded once for all records; acc[r] collects record r
// (rows g, g + 8 x tokens 2t, 2t + 1 of lane (g, t)).
template <typename T, typename S, int NREC, bool G32>
DEVI void pm_offset(const uint8_t* st, const TileGeom& tg, int pb, int pe, int lane,
                    const uint8_t* xsh, uint32_t pitch, const float2* gsum, bool xon,
                    float (&acc)[NREC][4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* xp = xsh + (uint32_t)g * pitch + (uint32_t)t * 16u + (uint32_t)pb * 128u;
  const uint8_t* wp = st + (((uint32_t)pb << 5) + lane) * 16u;
  int p = pb;
  while (p < pe) {
    if (G32) {
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (xon) {
        xa = *reinterpret_cast<const uint4*>(xp);
        xb = *reinterpret_cast<const uint4*>(xp + 64);
      }
      const float4 g0 = *reinterpret_cast<const float4*>(gsum + (2 * p) * 8 + 2 * t);
      const float4 g1 = *reinterpret_cast<const float4*>(gsum + (2 * p + 1) * 8 + 2 * t);
#pragma unroll
      for (int r = 0; r < NREC; ++r) {
        const uint8_t* rec = st + (uint32_t)r * tg.rec_bytes;
        const uint4 w = *reinterpret_cast<const uint4*>(wp + (uint32_t)r * tg.rec_bytes);
        float d0[4], d1[4];
        zero4(d0);
        zero4(d1);
        mma_window<T>(d0, d1, w.x, w.y, xa);
        flush_group<S>(acc[r], d0, d1, rec, tg, 2 * p, g, g0, 1.f, 1.f);
        zero4(d0);
        zero4(d1);
        mma_window<T>(d0, d1, w.z, w.w, xb);
        flush_group<S>(acc[r], d0, d1, rec, tg, 2 * p + 1, g, g1, 1.f, 1.f);
      }
      ++p;
      xp += 128;
      wp += 512;
    } else {
      const int grp = p >> tg.gshift;
      int pend = (grp + 1) << tg.gshift;
      if (pend > pe) pend = pe;
      float d0[NREC][4], d1[NREC][4];
#pragma unroll
      for (int r = 0; r < NREC; ++r) {
        zero4(d0[r]);
        zero4(d1[r]);
      }
      float4 gs = make_float4(0.f, 0.f, 0.f, 0.f);
      for (; p < pend; ++p, xp += 128, wp += 512) {
        const float4 gp = *reinterpret_cast<const float4*>(gsum + p * 8 + 2 * t);
        gs.x += gp.x;
        gs.y += gp.y;
        gs.z += gp.z;
        gs.w += gp.w;
        uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
        if (xon) {
          xa = *reinterpret_cast<const uint4*>(xp);
          xb = *reinterpret_cast<const uint4*>(xp + 64);
        }
#pragma unroll
        for (int r = 0; r < NREC; ++r) {
          const uint4 w = *reinterpret_cast<const uint4*>(wp + (uint32_t)r * tg.rec_bytes);
          mma_window<T>(d0[r], d1[r], w.x, w.y, xa);
          mma_window<T>(d0[r], d1[r], w.z, w.w, xb);
        }
      }
#pragma unroll
      for (int r = 0; r < NREC; ++r)
        flush_group<S>(acc[r], d0[r], d1[r], st + (uint32_t)r * tg.rec_bytes, tg, grp, g, gs, 1.f,
                       1.f);
    }
  }
}

// First MMA of a fresh accumulator: D = A B (no accumulator input).
template <typename T>
DEVI void mma_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                    uint32_t b1) {
  d[0] = d[1] = d[2] = d[3] = 0.f;
  MmaOp<T>::run(d, a0, a1, a2, a3, b0, b1);
}

// pm_offset for the common fixed geometry: the 16 warps each take PPW pairs
// (npairs == 16 PPW), a whole number of groups of PPG pairs, fully unrolled, one
// accumulator chain per record.
template <typename T, typename S, int NREC, int PPW, int PPG>
DEVI void pm_fixed(const uint8_t* st, const TileGeom& tg, int warp, int lane, const uint8_t* xsh,
                   uint32_t pitch, const float2* gsum, bool xon, float (&acc)[NREC][4]) {
  static_assert(PPW % PPG == 0, "warp ranges must hold whole groups");
  const int g = lane >> 2, t = lane & 3;
  const int pb = warp * PPW;
  const uint8_t* xp = xsh + (uint32_t)g * pitch + (uint32_t)t * 16u + (uint32_t)pb * 128u;
  const uint8_t* wp = st + (((uint32_t)pb << 5) + lane) * 16u;
  const float2* gp = gsum + pb * 8 + 2 * t;
#pragma unroll
  for (int gi = 0; gi < PPW / PPG; ++gi) {
    float d[NREC][4];
    float4 gs = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < PPG; ++k) {
      const int pi = gi * PPG + k;
      const float4 gq = *reinterpret_cast<const float4*>(gp + pi * 8);
      gs.x += gq.x;
      gs.y += gq.y;
      gs.z += gq.z;
      gs.w += gq.w;
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (xon) {
        xa = *reinterpret_cast<const uint4*>(xp + pi * 128);
        xb = *reinterpret_cast<const uint4*>(xp + pi * 128 + 64);
      }
#pragma unroll
      for (int r = 0; r < NREC; ++r) {
        const uint4 w = *reinterpret_cast<const uint4*>(wp + (uint32_t)r * tg.rec_bytes + pi * 512);
        uint32_t A[4], B[4];
        DqOff<T>::expand(w.x, w.y, A, B);
        if (k == 0)
          mma_first<T>(d[r], A[0], A[1], A[2], A[3], xa.x, xa.y);
        else
          MmaOp<T>::run(d[r], A[0], A[1], A[2], A[3], xa.x, xa.y);
        MmaOp<T>::run(d[r], B[0], B[1], B[2], B[3], xa.z, xa.w);
        DqOff<T>::expand(w.z, w.w, A, B);
        MmaOp<T>::run(d[r], A[0], A[1], A[2], A[3], xb.x, xb.y);
        MmaOp<T>::run(d[r], B[0], B[1], B[2], B[3], xb.z, xb.w);
      }
    }
    const int grp = (pb + gi * PPG) / PPG;
    const float zero4v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < NREC; ++r)
      flush_group<S>(acc[r], d[r], zero4v, st + (uint32_t)r * tg.rec_bytes, tg, grp, g, gs, 1.f, 1.f);
  }
}

// rm_offset for records whose pairs form whole groups of PPG pairs (npairs % PPG
// == 0): the items are (record, group), dealt round-robin to the 16 warps, each
// group's pairs fully unrolled with one accumulator chain.
template <typename T, typename S, int PPG>
DEVI void rm_grouped(const uint8_t* st, const TileGeom& tg, int nrec, int warp, int lane,
                     const uint8_t* xd, uint32_t xpitch, int rows_per_unit, const float2* gsum,
                     int gr_stride, const float* colw, bool xon, float (&acc)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const int gpr = tg.npairs / PPG;  // groups per record
  for (int it = warp; it < nrec * gpr; it += kCW) {
    const int us = it / gpr, grp = it - us * gpr;
    const uint8_t* rec = st + (uint32_t)us * tg.rec_bytes;
    const int p0 = grp * PPG;
    const uint8_t* xrow =
        xd + (uint32_t)(us * rows_per_unit + g) * xpitch + (uint32_t)t * 16u + (uint32_t)p0 * 128u;
    const uint8_t* wp = rec + (((uint32_t)p0 << 5) + lane) * 16u;
    const float2* gp = gsum + (size_t)us * gr_stride * 8 + p0 * 8 + 2 * t;
    float d[4];
    float4 gs = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < PPG; ++k) {
      const float4 gq = *reinterpret_cast<const float4*>(gp + k * 8);
      gs.x += gq.x;
      gs.y += gq.y;
      gs.z += gq.z;
      gs.w += gq.w;
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (xon) {
        xa = *reinterpret_cast<const uint4*>(xrow + k * 128);
        xb = *reinterpret_cast<const uint4*>(xrow + k * 128 + 64);
      }
      const uint4 w = *reinterpret_cast<const uint4*>(wp + k * 512);
      uint32_t A[4], B[4];
      DqOff<T>::expand(w.x, w.y, A, B);
      if (k == 0)
        mma_first<T>(d, A[0], A[1], A[2], A[3], xa.x, xa.y);
      else
        MmaOp<T>::run(d, A[0], A[1], A[2], A[3], xa.x, xa.y);
      MmaOp<T>::run(d, B[0], B[1], B[2], B[3], xa.z, xa.w);
      DqOff<T>::expand(w.z, w.w, A, B);
      MmaOp<T>::run(d, A[0], A[1], A[2], A[3], xb.x, xb.y);
      MmaOp<T>::run(d, B[0], B[1], B[2], B[3], xb.z, xb.w);
    }
    const float zero4v[4] = {0.f, 0.f, 0.f, 0.f};
    flush_group<S>(acc, d, zero4v, rec, tg, grp, g, gs, colw[us * 8 + 2 * t], colw[us * 8 + 2 * t + 1]);
  }
}

// Record-major walk over items [lo, hi) of a stage whose records each have their
// own activation rows (the MoE down projection: record us = unit us, rows
// us * rows_per_unit + token): item = (record, column pair), record-major.  gsum is
// [record][gr_stride pairs (windows when G32)][8 tokens]; colw [record][8] weights
// token columns.
template <typename T, typename S, bool G32>
DEVI void rm_offset(const uint8_t* st, const TileGeom& tg, int lo, int hi, int lane,
                    const uint8_t* xd, uint32_t xpitch, int rows_per_unit, const float2* gsum,
                    int gr_stride, const float* colw, bool xon, float (&acc)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const int np = tg.npairs;
  int us = lo / np, pp = lo - us * np;
  int it = lo;
  while (it < hi) {
    const uint8_t* rec = st + (uint32_t)us * tg.rec_bytes;
    const uint8_t* xrow =
        xd + (uint32_t)(us * rows_per_unit + g) * xpitch + (uint32_t)t * 16u + (uint32_t)pp * 128u;
    const uint8_t* wp = rec + (((uint32_t)pp << 5) + lane) * 16u;
    const float w0 = colw[us * 8 + 2 * t], w1 = colw[us * 8 + 2 * t + 1];
    const float2* gsu = gsum + (size_t)us * gr_stride * 8;
    if (G32) {
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (xon) {
        xa = *reinterpret_cast<const uint4*>(xrow);
        xb = *reinterpret_cast<const uint4*>(xrow + 64);
      }
      const uint4 w = *reinterpret_cast<const uint4*>(wp);
      float d0[4], d1[4];
      zero4(d0);
      zero4(d1);
      mma_window<T>(d0, d1, w.x, w.y, xa);
      flush_group<S>(acc, d0, d1, rec, tg, 2 * pp, g,
                     *reinterpret_cast<const float4*>(gsu + (2 * pp) * 8 + 2 * t), w0, w1);
      zero4(d0);
      zero4(d1);
      mma_window<T>(d0, d1, w.z, w.w, xb);
      flush_group<S>(acc, d0, d1, rec, tg, 2 * pp + 1, g,
                     *reinterpret_cast<const float4*>(gsu + (2 * pp + 1) * 8 + 2 * t), w0, w1);
      ++it;
      if (++pp == np) {
        pp = 0;
        ++us;
      }
    } else {
      const int grp = pp >> tg.gshift;
      int pend = (grp + 1) << tg.gshift;
      if (pend > np) pend = np;
      int n_it = pend - pp;
      if (n_it > hi - it) n_it = hi - it;
      float d0[4], d1[4];
      zero4(d0);
      zero4(d1);
      float4 gs = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < n_it; ++k, xrow += 128, wp += 512) {
        const float4 gp = *reinterpret_cast<const float4*>(gsu + (pp + k) * 8 + 2 * t);
        gs.x += gp.x;
        gs.y += gp.y;
        gs.z += gp.z;
        gs.w += gp.w;
        uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
        if (xon) {
          xa = *reinterpret_cast<const uint4*>(xrow);
          xb = *reinterpret_cast<const uint4*>(xrow + 64);
        }
        const uint4 w = *reinterpret_cast<const uint4*>(wp);
        mma_window<T>(d0, d1, w.x, w.y, xa);
        mma_window<T>(d0, d1, w.z, w.w, xb);
      }
      flush_group<S>(acc, d0, d1, rec, tg, grp, g, gs, w0, w1);
      it += n_it;
      pp += n_it;
      if (pp == np) {
        pp = 0;
        ++us;
      }
    }
  }
}

// Cross-warp reduction of one output tile (16 rows x 8 columns; with `two`, a second
// set for record 1).  On return (after a consumer barrier) threads tid < 128 hold
// the sums for row r = tid & 15, column n = tid >> 4 in v (and v2).
DEVI void reduce_tile(float* red, const float (&acc0)[4], const float (&acc1)[4], bool two,
                      int tid, int warp, int lane, float& v, float& v2) {
#pragma unroll
  for (int r = 0; r < 4; ++r) red[(warp * 8 + r) * 32 + lane] = acc0[r];
  if (two) {
#pragma unroll
    for (int r = 0; r < 4; ++r) red[(warp * 8 + 4 + r) * 32 + lane] = acc1[r];
  }
  named_bar_sync(1, kConsumers);
  v = 0.f;
  v2 = 0.f;
  if (tid < 128) {
    const int n = tid >> 4, r = tid & 15;
    const int gl = (r & 7) * 4 + (n >> 1);
    const int ri = (r >> 3) * 2 + (n & 1);
#pragma unroll
    for (int w = 0; w < kCW; ++w) {
      v += red[(w * 8 + ri) * 32 + gl];
      if (two) v2 += red[(w * 8 + 4 + ri) * 32 + gl];
    }
  }
}

}  // namespace duplex
