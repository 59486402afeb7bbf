// dcnv2_kernels.cuh — sm_100a DCNv2 forward kernels.
//
// The reference computes the forward in three launches per image (src/dcn_plugin.cpp:135-174):
// a deformable im2col that writes the column matrix [C*K*K, Ho*Wo] to HBM
// (src/dcn_kernel.cu:138-240), a cuBLAS GEMM, and a bias/scale pass (:168-178, :208-216,
// :249-257). Here one persistent, warp-specialised implicit-GEMM kernel per precision does all
// of it; the column matrix exists only as 128-byte-swizzled shared-memory tiles:
//
//   warp 0       producer: bulk-copies the pre-swizzled weight tile of each K-block into smem
//   warp 1       MMA issuer: tcgen05.mma (kind::f16 / kind::i8 / kind::tf32) into TMEM,
//                accumulator double-buffered so the epilogue overlaps the next tile
//   warps 2-5    epilogue: tcgen05.ld from TMEM, + bias (x x_scale*w_scale for int8), store y
//   warps 6-21   samplers: bilinear x mask samples of 128 output pixels x one K-block, written
//                straight into the A-operand tile (one 16-byte chunk of channels per thread)
//
// GEMM view per tile: D[128 pixels, O] = A[128 pixels, C*K*K] * B[O, C*K*K]^T. K is ordered
// (deformable group g, channel block, tap t): one K-block has one sampling geometry per pixel,
// and the K*K consecutive K-blocks of a channel block read one shared-memory window of x (a
// TMA box of whole rows of the channels-last copy, double-buffered), so most corner fetches are
// 16-byte shared-memory loads of 8 fp16 / 16 int8 / 4 fp32 channels. The corner weights of a
// (pixel, tap, group) are computed once per tile and reused for every channel block.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dcnv2.h"
#include "ptx_sm100.cuh"

namespace dcnv2 {

enum Prec : int { PREC_F32 = 0, PREC_F16 = 1, PREC_I8 = 2 };

constexpr int kTileM = 128;            // output pixels per tile (MMA M, TMEM lanes)
constexpr int kRowBytes = 128;         // bytes of one operand row per K-block (128-byte swizzle)
constexpr int kATileBytes = kTileM * kRowBytes;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;
constexpr int kNumEpiWarps = 4;
constexpr int kSampWarp0 = kEpiWarp0 + kNumEpiWarps;
constexpr int kNumSampWarps = 16;
constexpr int kThreads = (kSampWarp0 + kNumSampWarps) * 32;  // 704
constexpr int kMaxStages = 8;
constexpr int kRowsPerSampThread = kTileM * 8 / (kNumSampWarps * 32);  // 2
constexpr int kSampRowStride = kNumSampWarps * 32 / 8;              // 64

template <int P> struct PrecTraits;
template <> struct PrecTraits<PREC_F16> {
  using X = __half;  // x, offset, mask, weight, bias, y
  using G = __half;  // offset / mask element
  using Y = __half;
  static constexpr int kElemBytes = 2, kChunkElems = 8, kBlockElems = 64;
  static constexpr int kNumATiles = 1, kNumBTiles = 1;
};
template <> struct PrecTraits<PREC_I8> {
  using X = int8_t;
  using G = float;
  using Y = float;
  static constexpr int kElemBytes = 1, kChunkElems = 16, kBlockElems = 128;
  static constexpr int kNumATiles = 1, kNumBTiles = 1;
};
template <> struct PrecTraits<PREC_F32> {
  using X = float;
  using G = float;
  using Y = float;
  static constexpr int kElemBytes = 4, kChunkElems = 4, kBlockElems = 32;
  static constexpr int kNumATiles = 2, kNumBTiles = 2;  // 3xTF32: hi and lo parts
};

struct FusedArgs {
  const uint8_t* x_nhwc;   // [N][H][W][C] channels-last copy of x
  const void* offset;      // [N][dg*2*T][Ho][Wo]
  const void* mask;        // [N][dg*T][Ho][Wo]
  const uint8_t* wpack;    // [cchunks][numKB][kNumBTiles][nrows][128 B], pre-swizzled; for a
                           // CTA pair each K-block is [rank][nsub][n_mma/2][128 B]
  const void* bias;        // [O] or null
  void* y;                 // [N][O][Ho][Wo]
  int* err;                // device error word
  int N, C, H, W, O, Ho, Wo, P;
  int K, T, stride, pad, dil, dg, Cg, CBg, numKB;
  int tiles_per_img, cchunks, num_tiles;  // tiles of 128 pixels (256 for a CTA pair)
  int n_mma, nsub, nrows, acc_bufs;
  int stages;
  uint32_t tmem_cols;
  uint32_t a_stage_bytes, b_stage_bytes;  // per CTA (a pair's CTA holds half of the B rows)
  float scale;             // int8: x_scale * w_scale
  int use_win;             // 1: corners come from a shared-memory window of x (TMA)
  int win_rows;            // rows of x in one window (all W columns, 128 bytes per pixel)
  int win_top;             // window top row = first output row of the tile * stride - win_top
  uint32_t win_bytes;      // win_rows * W * 128
  uint32_t win_stride;     // distance of the two window buffers (win_bytes rounded up to 1 KB)
  int a_stages, b_stages;  // A operand in TMEM: A ring (TMEM) and B ring (shared memory) depths
  int tap_pairs;           // int8, 64-channel groups: K-block = taps (2i, 2i+1) x 64 channels
  int precise;             // fp16: fp32 sampler arithmetic
  int tf32_single;         // fp32: hi*hi only (plain TF32)
  uint32_t epi_off;        // A-in-shared-memory kernel, fp32 output: byte offset of the
                           // epilogue's TMA-store staging boxes from the barrier block (0: direct
                           // stores of y)
  unsigned long long timeout_ns;
};

// ------------------------------------------------------------------ bounded mbarrier wait
// Waits for the phase of `bar` with the given parity. Gives up after timeout_ns (sets the CTA
// abort flag and the device error word) or as soon as another role of this CTA has aborted;
// both are checked every 16 tries so that a waiting warp issues few instructions.
// SLEEP_NS > 0 adds a nanosleep between tries; SLEEP_NS < 0 (kSuspend) lets the hardware suspend
// the thread until the phase completes; 0 spins (the MMA issuer, whose wake-up latency is on the
// critical path). Waiting warps that do not spin leave the issue slots to the working ones.
// CL selects a cluster-scope acquire (barriers that the peer CTA of a pair arrives on).
constexpr int kSuspend = -1;
struct WaitCtx {
  unsigned long long timeout_ns;
  int* err;                  // device error word
  volatile int* abort_flag;  // this CTA's abort flag (shared memory)
};
template <int SLEEP_NS = 0, bool CL = false>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                         int code) {
  if (CL ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t n = 1;; ++n) {
    if constexpr (SLEEP_NS > 0) __nanosleep(static_cast<unsigned>(SLEEP_NS));
    if constexpr (CL) {
      if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
    } else if constexpr (SLEEP_NS < 0) {
      if (ptx::mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    } else {
      if (ptx::mbar_try_wait(bar, parity)) return true;
    }
    if ((n & 15u) == 0) {
      if (*w.abort_flag) return false;
      if (ptx::global_timer_ns() - t0 > w.timeout_ns) {
        *w.abort_flag = 1;
        atomicOr(w.err, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void decode_tile(const FusedArgs& a, int tile, int& img, int& pt,
                                            int& cc) {
  cc = tile % a.cchunks;
  const int r = tile / a.cchunks;
  pt = r % a.tiles_per_img;
  img = r / a.tiles_per_img;
}

// Geometry of one (pixel, tap, group): corner weights (mask folded in, zero when a corner is
// outside the image or the sample centre is outside (-1, H) x (-1, W)) and the element offsets
// of the four corner pixels inside the channels-last image (clamped, always readable).
// Same rules as bilinear<T> in the reference (src/dcn_kernel.cu:19-30); the mask product is
// applied to each corner weight instead of to the sum.
struct Geom {
  float a[4];
  int off[4];
};

__device__ __forceinline__ Geom make_geom(const FusedArgs& a, bool valid, int base_h,
                                          int base_w, float dh, float dw, float m) {
  Geom g;
  const float hf = __fadd_rn(static_cast<float>(base_h), dh);
  const float wf = __fadd_rn(static_cast<float>(base_w), dw);
  const bool inside = valid && !(hf <= -1.f || hf >= static_cast<float>(a.H) || wf <= -1.f ||
                                 wf >= static_cast<float>(a.W));
  const float h0f = floorf(hf), w0f = floorf(wf);
  const int h0 = inside ? static_cast<int>(h0f) : 0;
  const int w0 = inside ? static_cast<int>(w0f) : 0;
  const float lh = __fsub_rn(hf, h0f), lw = __fsub_rn(wf, w0f);
  const float hh = __fsub_rn(1.f, lh), hw = __fsub_rn(1.f, lw);
  const bool hl_ok = h0 >= 0, wl_ok = w0 >= 0;
  const bool hh_ok = h0 + 1 <= a.H - 1, wh_ok = w0 + 1 <= a.W - 1;
  g.a[0] = (inside && hl_ok && wl_ok) ? __fmul_rn(m, __fmul_rn(hh, hw)) : 0.f;
  g.a[1] = (inside && hl_ok && wh_ok) ? __fmul_rn(m, __fmul_rn(hh, lw)) : 0.f;
  g.a[2] = (inside && hh_ok && wl_ok) ? __fmul_rn(m, __fmul_rn(lh, hw)) : 0.f;
  g.a[3] = (inside && hh_ok && wh_ok) ? __fmul_rn(m, __fmul_rn(lh, lw)) : 0.f;
  const int hc0 = min(max(h0, 0), a.H - 1), hc1 = min(max(h0 + 1, 0), a.H - 1);
  const int wc0 = min(max(w0, 0), a.W - 1), wc1 = min(max(w0 + 1, 0), a.W - 1);
  g.off[0] = (hc0 * a.W + wc0) * a.C;
  g.off[1] = (hc0 * a.W + wc1) * a.C;
  g.off[2] = (hc1 * a.W + wc0) * a.C;
  g.off[3] = (hc1 * a.W + wc1) * a.C;
  return g;
}

// Corner c of make_geom alone (0: (h0,w0), 1: (h0,w0+1), 2: (h0+1,w0), 3: (h0+1,w0+1)), with
// the same operations in the same order, so weight and offset are bit-identical to make_geom's.
__device__ __forceinline__ void make_corner(const FusedArgs& a, bool valid, int base_h,
                                            int base_w, float dh, float dw, float m, int c,
                                            float& wt, int& off) {
  const float hf = __fadd_rn(static_cast<float>(base_h), dh);
  const float wf = __fadd_rn(static_cast<float>(base_w), dw);
  const bool inside = valid && !(hf <= -1.f || hf >= static_cast<float>(a.H) || wf <= -1.f ||
                                 wf >= static_cast<float>(a.W));
  const float h0f = floorf(hf), w0f = floorf(wf);
  const int h0 = inside ? static_cast<int>(h0f) : 0;
  const int w0 = inside ? static_cast<int>(w0f) : 0;
  const float lh = __fsub_rn(hf, h0f), lw = __fsub_rn(wf, w0f);
  const float hh = __fsub_rn(1.f, lh), hw = __fsub_rn(1.f, lw);
  const int dy = c >> 1, dx = c & 1;
  const float fy = dy ? lh : hh, fx = dx ? lw : hw;
  const int hc = h0 + dy, wc = w0 + dx;
  const bool ok = inside && hc >= 0 && hc <= a.H - 1 && wc >= 0 && wc <= a.W - 1;
  wt = ok ? __fmul_rn(m, __fmul_rn(fy, fx)) : 0.f;
  off = (min(max(hc, 0), a.H - 1) * a.W + min(max(wc, 0), a.W - 1)) * a.C;
}

__device__ __forceinline__ float load_geom_value(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float load_geom_value(const float* p) { return __ldg(p); }

__device__ __forceinline__ uint32_t h2_bits(__half2 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ __half2 bits_h2(uint32_t v) {
  return *reinterpret_cast<__half2*>(&v);
}

// ---- per-precision chunk computation: 4 corner vectors -> one 16-byte operand chunk ----
// fp16 fast path: packed half2 arithmetic, weights rounded to fp16.
__device__ __forceinline__ uint32_t f16_mix_fast(uint32_t a0, uint32_t a1, uint32_t a2,
                                                 uint32_t a3, uint32_t x0, uint32_t x1,
                                                 uint32_t x2, uint32_t x3) {
  __half2 v = __hmul2(bits_h2(a0), bits_h2(x0));
  v = __hfma2(bits_h2(a1), bits_h2(x1), v);
  v = __hfma2(bits_h2(a2), bits_h2(x2), v);
  v = __hfma2(bits_h2(a3), bits_h2(x3), v);
  return h2_bits(v);
}
// Same mix with the (duplicated) fp16 weights as __half2 operands.
__device__ __forceinline__ uint32_t f16_mix_h2(__half2 a0, __half2 a1, __half2 a2, __half2 a3,
                                               uint32_t x0, uint32_t x1, uint32_t x2,
                                               uint32_t x3) {
  __half2 v = __hmul2(a0, bits_h2(x0));
  v = __hfma2(a1, bits_h2(x1), v);
  v = __hfma2(a2, bits_h2(x2), v);
  v = __hfma2(a3, bits_h2(x3), v);
  return h2_bits(v);
}
// fp16 precise path: fp32 arithmetic, one rounding to fp16 per column value.
__device__ __forceinline__ uint32_t f16_mix_precise(const float (&a)[4], uint32_t x0,
                                                    uint32_t x1, uint32_t x2, uint32_t x3) {
  const float2 f0 = __half22float2(bits_h2(x0)), f1 = __half22float2(bits_h2(x1));
  const float2 f2 = __half22float2(bits_h2(x2)), f3 = __half22float2(bits_h2(x3));
  float lo = __fmul_rn(a[0], f0.x), hi = __fmul_rn(a[0], f0.y);
  lo = __fmaf_rn(a[1], f1.x, lo); hi = __fmaf_rn(a[1], f1.y, hi);
  lo = __fmaf_rn(a[2], f2.x, lo); hi = __fmaf_rn(a[2], f2.y, hi);
  lo = __fmaf_rn(a[3], f3.x, lo); hi = __fmaf_rn(a[3], f3.y, hi);
  return h2_bits(__floats2half2_rn(lo, hi));
}
// ---- int8 column requantisation (fixed point, exact in integers) ----
// A DCNv2 int8 column value is the bilinear sample of int8 x rounded to an integer:
//   m' = clamp(m, 0, 1)        (mask; NaN -> 0), corner weights a_k = m' * fy_k * fx_k (fp32)
//   w_k = min(rint(a_k * 2^16), 65535)                                          (u16)
//   c   = floor((sum_k w_k * x_k + 2^15) / 2^16)                 (in [-128, 127] always)
// |c - m' * bilinear(x)| <= 0.5 + 2^-7. dp2a forms the 2-term products and sums exactly; the
// column byte is byte 2 of the 32-bit sum, so nothing is converted to or from floating point.
__device__ __forceinline__ float i8_mask(float m) { return fminf(fmaxf(m, 0.f), 1.f); }
__device__ __forceinline__ uint32_t i8_weight(float a) {
  const uint32_t w = __float2uint_rn(__fmul_rn(a, 65536.f));  // NaN, a <= 0 -> 0
  return w < 65535u ? w : 65535u;
}
// Packed weight pairs (w0 | w1 << 16) and (w2 | w3 << 16).
__device__ __forceinline__ void i8_weight_pairs(const float (&a)[4], uint32_t& w01, uint32_t& w23) {
  w01 = i8_weight(a[0]) | (i8_weight(a[1]) << 16);
  w23 = i8_weight(a[2]) | (i8_weight(a[3]) << 16);
}
__device__ __forceinline__ int dp2a_lo_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// One word of 4 int8 channels from the same word of the 4 corners.
__device__ __forceinline__ uint32_t i8_mix_fx(uint32_t w01, uint32_t w23, uint32_t x0, uint32_t x1,
                                              uint32_t x2, uint32_t x3) {
  // corner bytes paired per channel: [x0.b0 x1.b0 x0.b1 x1.b1] and [x0.b2 x1.b2 x0.b3 x1.b3]
  const uint32_t t01l = __byte_perm(x0, x1, 0x5140), t01h = __byte_perm(x0, x1, 0x7362);
  const uint32_t t23l = __byte_perm(x2, x3, 0x5140), t23h = __byte_perm(x2, x3, 0x7362);
  const int s0 = dp2a_lo_us(w23, t23l, dp2a_lo_us(w01, t01l, 32768));
  const int s1 = dp2a_hi_us(w23, t23l, dp2a_hi_us(w01, t01l, 32768));
  const int s2 = dp2a_lo_us(w23, t23h, dp2a_lo_us(w01, t01h, 32768));
  const int s3 = dp2a_hi_us(w23, t23h, dp2a_hi_us(w01, t01h, 32768));
  const uint32_t p01 = __byte_perm(static_cast<uint32_t>(s0), static_cast<uint32_t>(s1), 0x0062);
  const uint32_t p23 = __byte_perm(static_cast<uint32_t>(s2), static_cast<uint32_t>(s3), 0x0062);
  return __byte_perm(p01, p23, 0x5410);
}
// Same from the fp32 corner weights (mask already clamped).
__device__ __forceinline__ uint32_t i8_mix_word(const float (&a)[4], uint32_t x0, uint32_t x1,
                                                uint32_t x2, uint32_t x3) {
  uint32_t w01, w23;
  i8_weight_pairs(a, w01, w23);
  return i8_mix_fx(w01, w23, x0, x1, x2, x3);
}
// fp32: v = a0*x0 (+ a1*x1 + a2*x2 + a3*x3 by fma), then the 3xTF32 split hi = tf32(v), lo = tf32(v - hi).
__device__ __forceinline__ void f32_mix(const float (&a)[4], const uint4& x0, const uint4& x1,
                                        const uint4& x2, const uint4& x3, uint4& hi, uint4& lo) {
  const uint32_t* p0 = &x0.x; const uint32_t* p1 = &x1.x;
  const uint32_t* p2 = &x2.x; const uint32_t* p3 = &x3.x;
  uint32_t* ph = &hi.x; uint32_t* pl = &lo.x;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float v = __fmul_rn(a[0], __uint_as_float(p0[e]));
    v = __fmaf_rn(a[1], __uint_as_float(p1[e]), v);
    v = __fmaf_rn(a[2], __uint_as_float(p2[e]), v);
    v = __fmaf_rn(a[3], __uint_as_float(p3[e]), v);
    const uint32_t h = ptx::cvt_rna_tf32(v);
    ph[e] = h;
    pl[e] = ptx::cvt_rna_tf32(__fsub_rn(v, __uint_as_float(h)));
  }
}

// ------------------------------------------------------------------ MMA issuer
// One thread on the critical path, in a function of its own (not inlined) so that its loop keeps
// its own registers whatever the sampler code around it needs. It spins on the stage barriers
// (the samplers suspend), keeps stage and phase counters incrementally and only patches the
// start-address field of the descriptors. The MMAs of a K-block are straight-line code: the
// number of sub-MMAs (NSUB) and the 3xTF32 choice are template parameters, because a runtime
// loop or branch around tcgen05.mma in this single-lane loop measured ~1.7x slower per K-block.
struct MmaParams {
  uint32_t a_base, b_base, a_stage_bytes, b_stage_bytes, tmem_base;
  uint32_t full_a, full_b, full_peer, empty, tfull, tempty, drain;
  int S, num_tiles, tile0, tstep, numKB, n_mma, nrows, acc_bufs;
  WaitCtx wc;
};

template <int PREC, bool PAIR, int NSUB, bool TF32_SINGLE>
__device__ __noinline__ void mma_issuer(const MmaParams mp) {
  const uint32_t m = PAIR ? 2 * kTileM : kTileM;
  uint32_t idesc;
  if (PREC == PREC_F16) idesc = ptx::make_idesc(1, 0, mp.n_mma, m);
  else if (PREC == PREC_I8) idesc = ptx::make_idesc(2, 1, mp.n_mma, m);
  else idesc = ptx::make_idesc(1, 2, mp.n_mma, m);
  const uint64_t desc0 = ptx::sw128_kmajor_desc(0);  // every field but the address
  const uint32_t acc_cols = static_cast<uint32_t>(mp.nrows);
  // B rows of one sub-MMA in this CTA's stage (a pair's CTA holds n_mma / 2 of them)
  const uint32_t sub_bytes = static_cast<uint32_t>(PAIR ? mp.n_mma / 2 : mp.n_mma) * kRowBytes;
  const uint32_t lo_bytes = static_cast<uint32_t>(mp.nrows) * kRowBytes;
  const WaitCtx& wc = mp.wc;
  const int S = mp.S, numKB = mp.numKB;
  int s = 0, acc = 0;
  uint32_t ph = 0, use = 0;
  bool ok = true;
  for (int tile = mp.tile0; tile < mp.num_tiles && ok; tile += mp.tstep) {
    if (!wait_bar<64, PAIR>(mp.tempty + 8 * acc, use ^ 1, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    ptx::tc_fence_after();
    const uint32_t d_base = mp.tmem_base + acc * acc_cols;
    for (int kb = 0; kb < numKB; ++kb) {
      if (!wait_bar(mp.full_a + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA) ||
          !wait_bar(mp.full_b + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA) ||
          (PAIR && !wait_bar<0, true>(mp.full_peer + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA))) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint64_t ad0 = desc0 | (((mp.a_base + s * mp.a_stage_bytes) >> 4) & 0x3FFFu);
      const uint64_t bd0 = desc0 | (((mp.b_base + s * mp.b_stage_bytes) >> 4) & 0x3FFFu);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ad = ad0 + 2 * k;  // +32 bytes per K-step (address field in 16 B)
        const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
        for (int sub = 0; sub < NSUB; ++sub) {
          const uint32_t d = d_base + sub * mp.n_mma;
          const uint64_t bd = bd0 + 2 * k + ((sub * sub_bytes) >> 4);
          if (PAIR) {
            if (PREC == PREC_F16) ptx::mma_f16_pair(d, ad, bd, idesc, accum);
            else ptx::mma_i8_pair(d, ad, bd, idesc, accum);
          } else if (PREC == PREC_F16) {
            ptx::mma_f16(d, ad, bd, idesc, accum);
          } else if (PREC == PREC_I8) {
            ptx::mma_i8(d, ad, bd, idesc, accum);
          } else {
            ptx::mma_tf32(d, ad, bd, idesc, accum);
            if (!TF32_SINGLE) {
              ptx::mma_tf32(d, ad, bd + (lo_bytes >> 4), idesc, 1u);
              ptx::mma_tf32(d, ad + (kATileBytes >> 4), bd, idesc, 1u);
            }
          }
        }
      }
      // frees this stage (in both CTAs of a pair) once its MMAs have read it
      if (PAIR) ptx::tc_commit_pair(mp.empty + 8 * s, 3);
      else ptx::tc_commit(mp.empty + 8 * s);
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    if (!ok) break;
    // accumulator ready for the epilogue(s)
    if (PAIR) ptx::tc_commit_pair(mp.tfull + 8 * acc, 3);
    else ptx::tc_commit(mp.tfull + 8 * acc);
    if (++acc == mp.acc_bufs) { acc = 0; use ^= 1u; }
  }
  if (PAIR) ptx::tc_commit_pair(mp.drain, 3);
  else ptx::tc_commit(mp.drain);
  wait_bar(mp.drain, 0, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
}

// ------------------------------------------------------------------ epilogue block
// 16 accumulator columns (output channels o_chunk + col ...) of one pixel per lane (pixel p,
// odd = p & 1 within the lane pair): + bias (int8: fma(float(acc), x_scale*w_scale, bias)), one
// rounding to the output type, stores of y (yimg = y of the tile's image). Bias comes from the
// fp32 copy in shared memory when `staged` (a global load per column would wait for L2 on every
// block: little L1 is left beside the shared memory these kernels use). When `paired` (P even,
// y aligned to two elements), lanes 2j and 2j+1 swap one value per channel pair so that each
// store covers the pixel pair (p - odd, p - odd + 1): the even lane stores the even channel, the
// odd lane the odd one. Layer sizes are read from the kernel arguments (not copied per tile:
// the kernels that call this have no registers to spare).
template <int PREC>
__device__ __forceinline__ void epilogue_block(const FusedArgs& args, const float* bias_smem,
                                               bool staged, bool paired,
                                               typename PrecTraits<PREC>::Y* yimg, int o_chunk,
                                               int p, int odd, const uint32_t (&r)[16], int col) {
  using YT = typename PrecTraits<PREC>::Y;
  const int o0 = o_chunk + col;
  const int pe = p - odd;
  float bo[16];
  if (staged) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 b4 = *reinterpret_cast<const float4*>(bias_smem + col + i);
      bo[i] = b4.x; bo[i + 1] = b4.y; bo[i + 2] = b4.z; bo[i + 3] = b4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int o = o0 + i < args.O ? o0 + i : args.O - 1;
      bo[i] = !args.bias ? 0.f
              : PREC == PREC_F16 ? __half2float(reinterpret_cast<const __half*>(args.bias)[o])
                                 : __ldg(reinterpret_cast<const float*>(args.bias) + o);
    }
  }
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (PREC == PREC_I8) v[i] = __fmaf_rn(__int2float_rn(static_cast<int>(r[i])), args.scale, bo[i]);
    else v[i] = __uint_as_float(r[i]) + bo[i];
  }
  if (paired) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float keep = odd ? v[2 * i + 1] : v[2 * i];
      const float send = odd ? v[2 * i] : v[2 * i + 1];
      const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
      const float lo = odd ? recv : keep, hi = odd ? keep : recv;
      const int o = o0 + 2 * i + odd;
      if (o < args.O && pe < args.P) {
        YT* dst = yimg + static_cast<size_t>(o) * args.P + pe;
        if (PREC == PREC_F16) *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(lo, hi);
        else *reinterpret_cast<float2*>(dst) = make_float2(lo, hi);
      }
    }
  } else if (p < args.P) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int o = o0 + i;
      if (o < args.O) {
        YT* dst = yimg + static_cast<size_t>(o) * args.P + p;
        if (PREC == PREC_F16) *reinterpret_cast<__half*>(dst) = __float2half_rn(v[i]);
        else *reinterpret_cast<float*>(dst) = v[i];
      }
    }
  }
}

// Same arithmetic as epilogue_block, written into a staging box of the epilogue's TMA store
// instead of y: box = [16 channels][32 pixels] of the output type at shared address `box`, lane
// = pixel (each channel row is 32 consecutive elements, so the lanes' stores are conflict-free).
template <int PREC>
__device__ __forceinline__ void epilogue_block_box(const FusedArgs& args, const float* bias_smem,
                                                   bool staged, int o_chunk,
                                                   const uint32_t (&r)[16], int col, uint32_t box,
                                                   int lane) {
  using YT = typename PrecTraits<PREC>::Y;
  const int o0 = o_chunk + col;
  float bo[16];
  if (staged) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 b4 = *reinterpret_cast<const float4*>(bias_smem + col + i);
      bo[i] = b4.x; bo[i + 1] = b4.y; bo[i + 2] = b4.z; bo[i + 3] = b4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int o = o0 + i < args.O ? o0 + i : args.O - 1;
      bo[i] = !args.bias ? 0.f
              : PREC == PREC_F16 ? __half2float(reinterpret_cast<const __half*>(args.bias)[o])
                                 : __ldg(reinterpret_cast<const float*>(args.bias) + o);
    }
  }
  const uint32_t at = box + static_cast<uint32_t>(lane) * sizeof(YT);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t row = at + static_cast<uint32_t>(i) * 32u * sizeof(YT);
    if (PREC == PREC_F16) {
      ptx::st_shared_u16(row, __half_as_ushort(__float2half_rn(__uint_as_float(r[i]) + bo[i])));
    } else if (PREC == PREC_I8) {
      ptx::st_shared_u32(row, __float_as_uint(
          __fmaf_rn(__int2float_rn(static_cast<int>(r[i])), args.scale, bo[i])));
    } else {
      ptx::st_shared_u32(row, __float_as_uint(__uint_as_float(r[i]) + bo[i]));
    }
  }
}

// ------------------------------------------------------------------ the fused kernel
// PAIR: launched as clusters of two CTAs that share each tile of 256 pixels (cta_group::2).
// Rank 0 (the leader) issues M = 256 MMAs reading rows 0-127 of A and B rows [0, N/2) from its own
// shared memory and rows 128-255 / [N/2, N) from the same offsets in rank 1; both CTAs sample their
// own 128 pixels, copy their half of the weights and run their own epilogue on their TMEM half.
// Rank 1's MMA thread relays "stage full" to the leader; the leader's completion commits arrive on
// the barriers of both CTAs.
template <int PREC, bool PRECISE, int KT, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    dcnv2_fused_kernel(const FusedArgs args, const __grid_constant__ CUtensorMap tmap_x,
                       const __grid_constant__ CUtensorMap tmap_y) {
  using TR = PrecTraits<PREC>;
  using GT = typename TR::G;
  using YT = typename TR::Y;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.stages;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + S * args.a_stage_bytes;
  uint8_t* w_smem = b_smem + S * args.b_stage_bytes;       // 2 x-window buffers (if used)
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_smem + (args.use_win ? 2 * args.win_bytes : 0));
  const uint32_t full_a = ptx::smem_addr(bars);          // [S]
  const uint32_t full_b = full_a + 8 * S;                // [S]
  const uint32_t empty = full_b + 8 * S;                 // [S]
  const uint32_t full_peer = empty + 8 * S;              // [S] (pair leader: stage full in rank 1)
  const uint32_t tfull = full_peer + 8 * S;              // [2]
  const uint32_t tempty = tfull + 16;                    // [2]
  const uint32_t drain = tempty + 16;                    // [1]
  const uint32_t win_full = drain + 8;                   // [2]
  const uint32_t win_empty = win_full + 16;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // bias of the (single) output-channel chunk as fp32, after the 512 bytes of barriers
  float* bias_smem = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512);
  const WaitCtx wc{args.timeout_ns, args.err, abort_flag};
  // Tile schedule: CTAs (pairs) stride over the tiles. pix_base(pt) is the first pixel of this
  // CTA's 128 rows in tile pt.
  const int rank = PAIR ? static_cast<int>(ptx::cluster_ctarank()) : 0;
  const int tile0 = PAIR ? static_cast<int>(ptx::cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(ptx::num_clusters_x()) : static_cast<int>(gridDim.x);
  auto pix_base = [&](int pt) { return pt * (PAIR ? 2 * kTileM : kTileM) + rank * kTileM; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(full_a + 8 * s, kNumSampWarps);
      ptx::mbar_init(full_b + 8 * s, 1);
      ptx::mbar_init(empty + 8 * s, 1);
      ptx::mbar_init(full_peer + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(tfull + 8 * i, 1);
      ptx::mbar_init(tempty + 8 * i, PAIR ? 2 * kNumEpiWarps : kNumEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(win_full + 8 * i, 1);
      ptx::mbar_init(win_empty + 8 * i, kNumSampWarps);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (args.cchunks == 1) {
    for (int i = threadIdx.x; i < args.nrows; i += blockDim.x) {
      float bv = 0.f;
      if (args.bias && i < args.O)
        bv = PREC == PREC_F16 ? __half2float(reinterpret_cast<const __half*>(args.bias)[i])
                              : reinterpret_cast<const float*>(args.bias)[i];
      bias_smem[i] = bv;
    }
  }
  if (warp == kMmaWarp) {
    if (PAIR) {
      ptx::tmem_alloc_pair(ptx::smem_addr(tmem_slot), args.tmem_cols);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_addr(tmem_slot), args.tmem_cols);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  if (PAIR) ptx::cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  else __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the setup above overlaps the tail of the kernel ahead (programmatic dependent launch); its
  // outputs (the channels-last x, packed weights, cleared error word) are read only from here
  ptx::griddep_wait();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer (weights)
    if (lane == 0) {
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t b_base = ptx::smem_addr(b_smem);
      // a K-block of packed weights holds both halves of a pair, this CTA copies its own
      const size_t kb_bytes = static_cast<size_t>(args.b_stage_bytes) * (PAIR ? 2 : 1);
      for (int tile = tile0; tile < args.num_tiles && ok; tile += tstep) {
        int img, pt, cc;
        decode_tile(args, tile, img, pt, cc);
        const uint8_t* src = args.wpack + static_cast<size_t>(cc) * args.numKB * kb_bytes +
                             static_cast<size_t>(rank) * args.b_stage_bytes;
        for (int kb = 0; kb < args.numKB; ++kb, ++it) {
          if (!wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc,
                                  DCNV2_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(full_b + 8 * s, args.b_stage_bytes);
          ptx::bulk_copy_g2s(b_base + s * args.b_stage_bytes,
                             src + static_cast<size_t>(kb) * kb_bytes,
                             args.b_stage_bytes, full_b + 8 * s);
          if (++s == S) { s = 0; ph ^= 1u; }
        }
      }
      // Wait for the copies still in flight (at most the last one per stage) before the CTA
      // can exit and release its shared memory.
      const int outstanding = it < S ? it : S;
      for (int j = 0; j < outstanding; ++j) {
        const int idx = it - 1 - j;
        wait_bar(full_b + 8 * (idx % S), (idx / S) & 1, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && (!PAIR || rank == 0)) {
      MmaParams mp;
      mp.a_base = ptx::smem_addr(a_smem);
      mp.b_base = ptx::smem_addr(b_smem);
      mp.a_stage_bytes = args.a_stage_bytes;
      mp.b_stage_bytes = args.b_stage_bytes;
      mp.tmem_base = tmem_base;
      mp.full_a = full_a; mp.full_b = full_b; mp.full_peer = full_peer; mp.empty = empty;
      mp.tfull = tfull; mp.tempty = tempty; mp.drain = drain;
      mp.S = S; mp.num_tiles = args.num_tiles; mp.tile0 = tile0; mp.tstep = tstep;
      mp.numKB = args.numKB; mp.n_mma = args.n_mma; mp.nrows = args.nrows;
      mp.acc_bufs = args.acc_bufs;
      mp.wc = wc;
      // nsub is 1 or 2 (at most 512 output channels per tile)
      if (args.nsub == 1) {
        if (PREC == PREC_F32 && args.tf32_single) mma_issuer<PREC, PAIR, 1, true>(mp);
        else mma_issuer<PREC, PAIR, 1, false>(mp);
      } else {
        if (PREC == PREC_F32 && args.tf32_single) mma_issuer<PREC, PAIR, 2, true>(mp);
        else mma_issuer<PREC, PAIR, 2, false>(mp);
      }
    } else if (PAIR && lane == 0) {
      // Rank 1 relay: once this CTA's A and B of a stage have landed, tell the leader.
      const uint32_t peer_full = ptx::mapa_shared(full_peer, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = tile0; tile < args.num_tiles && ok; tile += tstep) {
        for (int kb = 0; kb < args.numKB; ++kb) {
          if (!wait_bar(full_a + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA) ||
              !wait_bar(full_b + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_cluster(peer_full + 8 * s);
          if (++s == S) { s = 0; ph ^= 1u; }
        }
      }
      // the leader's last commit: every MMA reading this CTA's memory or TMEM has completed
      wait_bar(drain, 0, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
    }
  } else if (warp < kSampWarp0) {
    // ------------------------------------------------------------ epilogue
    // Per 16 accumulator columns: tcgen05.ld (the next block's load overlaps this block's
    // stores), then epilogue_block (+ bias from shared memory, convert, paired stores). With
    // 512 output channels the accumulator fills the TMEM, so the next tile's MMAs wait for this
    // drain: its speed is on the critical path.
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t acc_cols = static_cast<uint32_t>(args.nrows);
    const bool paired = (args.P % 2) == 0 &&
                        (reinterpret_cast<uintptr_t>(args.y) % (2 * sizeof(YT))) == 0;
    const bool staged = args.cchunks == 1;
    const int odd = lane & 1;
    // TMA-store path (fp32 outputs): two staging boxes per epilogue warp after the staged bias
    constexpr uint32_t kEpiBoxBytes = 16u * 32u * sizeof(YT);
    const bool y_tma = PREC != PREC_F16 && args.epi_off != 0;
    const uint32_t epi_slots = ptx::smem_addr(reinterpret_cast<uint8_t*>(bars) + args.epi_off);
    int nbox = 0;
    int tl = 0;
    for (int tile = tile0; tile < args.num_tiles; tile += tstep, ++tl) {
      const int acc = tl % args.acc_bufs;
      const uint32_t ph = (tl / args.acc_bufs) & 1;
      // Warp-uniform outcome: every lane must take part in the tcgen05.ld below or none.
      const bool got =
          wait_bar<256>(tfull + 8 * acc, ph, wc, DCNV2_DEVERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      ptx::tc_fence_after();
      int img, pt, cc;
      decode_tile(args, tile, img, pt, cc);
      const int p = pix_base(pt) + q * 32 + lane;
      const int o_chunk = cc * args.nrows;
      YT* yimg = reinterpret_cast<YT*>(args.y) + static_cast<size_t>(img) * args.O * args.P;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * acc_cols;
      const int ncols = args.O - o_chunk < args.nrows ? args.O - o_chunk : args.nrows;
      uint32_t ra[16], rb[16];
      if (y_tma) {
        // Per 16 columns: the converted [16 channels][32 pixels] box of this warp into one of
        // its two staging slots, then one TMA store by lane 0 (the parts past P or O are not
        // written). A slot is rewritten once the store issued from it two boxes earlier has
        // read it. TMEM is released after the last tcgen05.ld, without waiting for the stores.
        const int x0 = p - lane;  // first pixel of this warp's 32
        auto box = [&](const uint32_t (&r)[16], int col) {
          if (lane == 0) ptx::bulk_wait_group_read<1>();
          __syncwarp();
          const uint32_t slot = epi_slots + static_cast<uint32_t>(2 * q + nbox) * kEpiBoxBytes;
          epilogue_block_box<PREC>(args, bias_smem, staged, o_chunk, r, col, slot, lane);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && x0 < args.P) {  // a warp wholly past the last pixel stores nothing
            ptx::tma_store_3d(&tmap_y, slot, x0, o_chunk + col, img);
            ptx::bulk_commit_group();
          }
          nbox ^= 1;
        };
        ptx::tmem_ld_32x32b_x16(taddr, ra);
        for (int col = 0; col < ncols; col += 32) {  // warp-uniform bounds
          ptx::tmem_wait_ld_regs(ra);
          if (col + 16 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 16, rb);
          box(ra, col);
          if (col + 16 < ncols) {
            ptx::tmem_wait_ld_regs(rb);
            if (col + 32 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 32, ra);
            box(rb, col + 16);
          }
        }
      } else {
        ptx::tmem_ld_32x32b_x16(taddr, ra);
        for (int col = 0; col < ncols; col += 32) {  // warp-uniform bounds
          ptx::tmem_wait_ld_regs(ra);
          if (col + 16 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 16, rb);
          epilogue_block<PREC>(args, bias_smem, staged, paired, yimg, o_chunk, p, odd, ra, col);
          if (col + 16 < ncols) {
            ptx::tmem_wait_ld_regs(rb);
            if (col + 32 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 32, ra);
            epilogue_block<PREC>(args, bias_smem, staged, paired, yimg, o_chunk, p, odd, rb,
                                 col + 16);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(tempty + 8 * acc, 0));
        else ptx::mbar_arrive(tempty + 8 * acc);
      }
    }
    // the TMA stores of y have been performed (and have read their boxes) before the CTA exits
    if (y_tma && lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  } else {
    // ------------------------------------------------------------ samplers
    // K order is (group g, channel block cbg, tap t). Thread (pixel slot ps, chunk j) fills rows
    // ps and ps + 64, 16-byte chunk j, of every A tile.
    // Geometry: the 8 lanes of a pixel slot own the 8 (row, corner) items of its two rows. Per
    // (tile, group) each lane computes its item for every tap once (registers; the taps are
    // unrolled when KT > 0) and per K-block the items of the current tap are shuffled to the 8
    // lanes. An item is the corner weight and its location: a pixel index inside the shared-memory
    // window of x (use_win: the 128-byte channel block of win_rows whole rows), or, when the
    // corner lies outside the window, its pixel index in the channels-last copy of x in global
    // memory. A corner outside the image has weight 0 and points at window / global pixel 0.
    // For the fp16 fast path an item packs weight (low 16 bits) and window pixel (high 16 bits,
    // 0xFFFF = not in the window) into one word. A K-block whose warp has only in-window items
    // and full channel chunks takes a straight-line path of shared-memory loads.
    // Each K-block issues its 8 corner loads before waiting for the A stage to be free.
    constexpr int EPC = TR::kChunkElems, KC = TR::kBlockElems, EB = TR::kElemBytes;
    constexpr int R = kRowsPerSampThread;
    constexpr bool kPacked = (PREC == PREC_F16 && !PRECISE);
    constexpr uint32_t kNoWin = 0xFFFFu;
    constexpr int kCache = KT > 0 ? KT : 1;
    static_assert(R * 4 == 8, "one (row, corner) item per lane of a pixel-slot group");
    const int st = threadIdx.x - kSampWarp0 * 32;
    const int sw = st >> 5;     // sampler warp
    const int j = st & 7;       // 16-byte chunk of the 128-byte row
    const int ps = st >> 3;     // pixel slot
    const int myr = j >> 2, myc = j & 3;
    const int grp = lane & ~7;
    const bool issuer = args.use_win && sw == 0 && lane == 0;  // issues the window loads
    const GT* offp = reinterpret_cast<const GT*>(args.offset);
    const GT* maskp = reinterpret_cast<const GT*>(args.mask);
    const uint32_t w_base = ptx::smem_addr(w_smem);
    const uint32_t a_base = ptx::smem_addr(a_smem);
    const int cb_per_tile = args.dg * args.CBg;
    const int T = KT > 0 ? KT : args.T;
    // this thread's two chunk positions inside an A stage (fixed for the whole kernel)
    uint32_t dst_off[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m_row = ps + kSampRowStride * r;
      dst_off[r] = m_row * kRowBytes + ((j ^ (m_row & 7)) << 4);
    }
    int s = 0;                  // A stage
    uint32_t ph = 0;            // its phase
    int cbi = 0;                // channel-block sequence number (window buffer = cbi & 1)
    int issued = 0;             // windows issued so far (issuer)
    bool ok = true;

    // Window load of channel block q of this CTA's sequence (issuer only): waits until buffer
    // q & 1 is released by all sampler warps (its use q - 2), then one 4-D TMA box.
    auto issue_window = [&](int q) -> bool {
      const int k = q / cb_per_tile, r = q - k * cb_per_tile;
      const int tl = tile0 + k * tstep;
      if (tl >= args.num_tiles) return true;
      const int g = r / args.CBg, cbg = r - g * args.CBg;
      int im, pt, cc;
      decode_tile(args, tl, im, pt, cc);
      const int row0 = (pix_base(pt) / args.Wo) * args.stride - args.win_top;
      const int b = q & 1;
      const uint32_t use = static_cast<uint32_t>(q >> 1) & 1u;
      if (!wait_bar<kSuspend>(win_empty + 8 * b, use ^ 1u, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER))
        return false;
      ptx::mbar_arrive_expect_tx(win_full + 8 * b, args.win_bytes);
      ptx::tma_load_4d(w_base + b * args.win_bytes, &tmap_x, (g * args.Cg + cbg * KC) * EB, 0,
                       row0, im, win_full + 8 * b);
      issued = q + 1;
      return true;
    };
    if (issuer) ok = issue_window(0) && issue_window(1);
    ok = __all_sync(0xffffffffu, ok);

    // L2 prefetch of the offsets and mask of tile `tl` (this CTA's pixels, every group): the
    // items of a tile are computed from them when it starts, one tile after the prefetch. Every
    // address lies inside the prefetched range.
    auto prefetch_geometry = [&](int tl) {
      if (tl >= args.num_tiles) return;
      int im, ptn, ccn;
      decode_tile(args, tl, im, ptn, ccn);
      const int p0 = pix_base(ptn);
      const int cnt = args.P - p0 < kTileM ? args.P - p0 : kTileM;
      if (cnt <= 0) return;
      const int bytes = cnt * static_cast<int>(sizeof(GT));
      const int lines = (bytes + 127) / 128 + 1;  // +1: the range may straddle one more line
      const int off_planes = 2 * args.T * args.dg;
      const int planes = off_planes + args.T * args.dg;
      for (int i = lane; i < planes * lines; i += 32) {
        const int pl = i / lines, ln = i - pl * lines;
        const GT* base = pl < off_planes
                             ? offp + (static_cast<size_t>(im) * off_planes + pl) * args.P + p0
                             : maskp + (static_cast<size_t>(im) * args.T * args.dg +
                                        (pl - off_planes)) * args.P + p0;
        const int at = ln * 128 < bytes - 1 ? ln * 128 : bytes - 1;
        ptx::prefetch_l2(reinterpret_cast<const uint8_t*>(base) + at);
      }
    };

    for (int tile = tile0; tile < args.num_tiles && ok; tile += tstep) {
      int img, pt, cc;
      decode_tile(args, tile, img, pt, cc);
      const int my_pix = pix_base(pt) + ps + kSampRowStride * myr;
      const bool my_val = my_pix < args.P;
      const int pcl = my_val ? my_pix : 0;
      const int oh = pcl / args.Wo, ow = pcl - (pcl / args.Wo) * args.Wo;
      const int my_bh = oh * args.stride - args.pad;
      const int my_bw = ow * args.stride - args.pad;
      const int row0 = (pix_base(pt) / args.Wo) * args.stride - args.win_top;
      const uint8_t* ximg = args.x_nhwc + static_cast<size_t>(img) * args.H * args.W * args.C * EB;
      if (sw == 0) prefetch_geometry(tile + tstep);

      // this lane's item of tap t: weight word (packed for the fp16 fast path) and global pixel
      // geometry value i of (group g) for this lane's pixel: i = 3t + {0: dh, 1: dw, 2: mask}
      auto geom = [&](int g, int i) -> float {
        const int t = i / 3, comp = i - 3 * t;
        const size_t ig = static_cast<size_t>(img) * args.dg + g;
        return comp < 2 ? load_geom_value(offp + (ig * 2 * args.T + 2 * t + comp) * args.P + my_pix)
                        : load_geom_value(maskp + (ig * args.T + t) * args.P + my_pix);
      };
      // this lane's item of tap t from the pixel's (dh, dw, m)
      auto item_from = [&](int t, float dh, float dw, float m, uint32_t& wword, int& gpix) {
        if (PREC == PREC_I8) m = i8_mask(m);
        const int ki = t / args.K, kj = t - ki * args.K;
        const float hf = __fadd_rn(static_cast<float>(my_bh + ki * args.dil), dh);
        const float wf = __fadd_rn(static_cast<float>(my_bw + kj * args.dil), dw);
        const bool inside = my_val && !(hf <= -1.f || hf >= static_cast<float>(args.H) ||
                                        wf <= -1.f || wf >= static_cast<float>(args.W));
        const float h0f = floorf(hf), w0f = floorf(wf);
        const int h0 = inside ? static_cast<int>(h0f) : 0;
        const int w0 = inside ? static_cast<int>(w0f) : 0;
        const float lh = __fsub_rn(hf, h0f), lw = __fsub_rn(wf, w0f);
        const float hh = __fsub_rn(1.f, lh), hw = __fsub_rn(1.f, lw);
        const int dy = myc >> 1, dx = myc & 1;
        const float fy = dy ? lh : hh, fx = dx ? lw : hw;
        const int hc = h0 + dy, wc = w0 + dx;
        const bool cok = inside && hc >= 0 && hc <= args.H - 1 && wc >= 0 && wc <= args.W - 1;
        const float wt = cok ? __fmul_rn(m, __fmul_rn(fy, fx)) : 0.f;
        gpix = cok ? hc * args.W + wc : 0;
        uint32_t wpix = kNoWin;  // pixel inside the window
        if (!cok) wpix = 0;
        else if (args.use_win && hc >= row0 && hc < row0 + args.win_rows)
          wpix = static_cast<uint32_t>((hc - row0) * args.W + wc);
        if (!args.use_win) wpix = kNoWin;
        if (kPacked) {
          // high half: byte offset of the pixel in the window (windows are at most 64 KB)
          const uint32_t hb = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(wt)));
          wword = hb | ((wpix != kNoWin ? wpix * kRowBytes : kNoWin) << 16);
        } else {
          wword = __float_as_uint(wt);
          gpix = (wpix != kNoWin) ? -static_cast<int>(wpix) - 1 : gpix;  // < 0: window pixel
        }
      };
      auto item = [&](int g, int t, uint32_t& wword, int& gpix) {
        float dh = 0.f, dw = 0.f, m = 0.f;
        if (my_val) {
          dh = geom(g, 3 * t);
          dw = geom(g, 3 * t + 1);
          m = geom(g, 3 * t + 2);
        }
        item_from(t, dh, dw, m, wword, gpix);
      };

      // No window (W too wide for one): for fp16 the cached item packs the corner's pixel index
      // in the image (< 2^16) beside its weight instead of a window offset (block-uniform).
      const bool gpacked = kPacked && !args.use_win && args.H * args.W <= 65536;
      for (int g = 0; g < args.dg && ok; ++g) {
        // items of every tap, computed once per (tile, group) for 3x3 kernels
        uint32_t cw[kCache];
        int cg[kCache];
        bool fast_g = false;
        if (KT > 0) {
          // The 4 lanes of a (pixel, row) share its 3*KT geometry values: lane c loads values
          // c, c+4, c+8, ... (one round trip of independent loads) and the rest are shuffled in.
          constexpr int kGeo = 3 * kCache, kPer = (kGeo + 3) / 4;
          float gv[kPer];
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const int i = 4 * q + myc;
            gv[q] = (my_val && i < kGeo) ? geom(g, i) : 0.f;
          }
          const int gl = lane & ~3;
          bool inwin = true;
#pragma unroll
          for (int t = 0; t < kCache; ++t) {
            const float dh = __shfl_sync(0xffffffffu, gv[(3 * t) >> 2], gl | ((3 * t) & 3));
            const float dw = __shfl_sync(0xffffffffu, gv[(3 * t + 1) >> 2], gl | ((3 * t + 1) & 3));
            const float m = __shfl_sync(0xffffffffu, gv[(3 * t + 2) >> 2], gl | ((3 * t + 2) & 3));
            item_from(t, dh, dw, m, cw[t], cg[t]);
            // in the window: packed word's high half, else a negative (window) location
            inwin = inwin && (kPacked ? ((cw[t] >> 16) != kNoWin) : (cg[t] < 0));
            if (gpacked) cw[t] = (cw[t] & 0xFFFFu) | (static_cast<uint32_t>(cg[t]) << 16);
          }
          // fp32 keeps the general path (two A tiles per K-block)
          fast_g = PREC != PREC_F32 && __all_sync(0xffffffffu, inwin);
        }
        const int gbase = g * args.Cg;
        for (int cbg = 0; cbg < args.CBg && ok; ++cbg) {
          const int b = cbi & 1;
          if (args.use_win) {
            const bool got = wait_bar<kSuspend>(win_full + 8 * b, static_cast<uint32_t>(cbi >> 1) & 1u,
                                      wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
          }
          const uint32_t win = w_base + b * args.win_bytes + j * 16;
          const int cig = cbg * KC + j * EPC;  // channel within the group
          const bool cvalid = cig < args.Cg;
          const bool all_valid = (cbg + 1) * KC <= args.Cg;  // block-uniform
          const uint8_t* gsrc = ximg + static_cast<size_t>(gbase + cig) * EB;
          if (kPacked && fast_g && all_valid) {
            // Fast path: every corner of every tap of this warp is in the window and every
            // chunk is full. Straight-line per tap: 8 shuffles, 8 shared loads and the mix run
            // before the stage is free; only the 2 stores and the arrive follow the wait (the
            // stage hand-off is the latency-critical loop of the pipeline).
#pragma unroll
            for (int tt = 0; tt < kCache; ++tt) {
              uint4 out[R];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                uint32_t wv[4];
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const uint32_t v = __shfl_sync(0xffffffffu, cw[tt], grp | (r * 4 + c));
                  wv[c] = v;                                   // fp16 weight in bits 0-15
                  xv[c] = ptx::ld_shared_v4(win + (v >> 16));  // window byte offset
                }
                const __half2 w0 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[0])));
                const __half2 w1 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[1])));
                const __half2 w2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[2])));
                const __half2 w3 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[3])));
                out[r].x = f16_mix_h2(w0, w1, w2, w3, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                out[r].y = f16_mix_h2(w0, w1, w2, w3, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                out[r].z = f16_mix_h2(w0, w1, w2, w3, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                out[r].w = f16_mix_h2(w0, w1, w2, w3, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
              }
              const bool got =
                  wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
              if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
              const uint32_t a_s = a_base + s * args.a_stage_bytes;
#pragma unroll
              for (int r = 0; r < R; ++r) ptx::st_shared_v4(a_s + dst_off[r], out[r]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(full_a + 8 * s);
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          } else if (!kPacked && PREC != PREC_F32 && fast_g && all_valid) {
            // Fast path of int8 and precise fp16: as above, with fp32 corner weights and window
            // byte offsets shuffled separately (same arithmetic as the general path).
#pragma unroll
            for (int tt = 0; tt < kCache; ++tt) {
              uint4 out[R];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float wf4[4];
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int src = grp | (r * 4 + c);
                  wf4[c] = __uint_as_float(__shfl_sync(0xffffffffu, cw[tt], src));
                  const int loc = __shfl_sync(0xffffffffu, cg[tt], src);  // -(window pixel) - 1
                  xv[c] = ptx::ld_shared_v4(win + static_cast<uint32_t>(-loc - 1) * kRowBytes);
                }
                if (PREC == PREC_I8) {
                  out[r].x = i8_mix_word(wf4, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[r].y = i8_mix_word(wf4, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[r].z = i8_mix_word(wf4, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[r].w = i8_mix_word(wf4, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                } else {
                  out[r].x = f16_mix_precise(wf4, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[r].y = f16_mix_precise(wf4, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[r].z = f16_mix_precise(wf4, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[r].w = f16_mix_precise(wf4, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                }
              }
              const bool got =
                  wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
              if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
              const uint32_t a_s = a_base + s * args.a_stage_bytes;
#pragma unroll
              for (int r = 0; r < R; ++r) ptx::st_shared_v4(a_s + dst_off[r], out[r]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(full_a + 8 * s);
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          } else if (KT > 0 && PREC == PREC_I8 && args.tap_pairs) {
            // int8 with 64-channel groups, no window: K-block i holds taps 2i (chunks 0-3) and
            // 2i+1 (chunks 4-7, zero past the last tap), so every lane loads and the group takes
            // 5 K-blocks instead of 9 half-empty ones. Lane j takes the items of its own tap.
            const uint32_t row_bytes = static_cast<uint32_t>(args.C) * EB;
            const bool hi = j >= 4;
            const uint8_t* psrc = ximg + static_cast<size_t>(gbase + (j & 3) * EPC) * EB;
#pragma unroll
            for (int pp = 0; pp < (kCache + 1) / 2; ++pp) {
              const int t0 = 2 * pp, t1 = 2 * pp + 1 < kCache ? 2 * pp + 1 : 2 * pp;
              const bool lane_valid = !(hi && 2 * pp + 1 >= kCache);
              uint4 out[R];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float wf4[4];
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int src = grp | (r * 4 + c);
                  const uint32_t w0 = __shfl_sync(0xffffffffu, cw[t0], src);
                  const uint32_t w1 = __shfl_sync(0xffffffffu, cw[t1], src);
                  const int g0 = __shfl_sync(0xffffffffu, cg[t0], src);
                  const int g1 = __shfl_sync(0xffffffffu, cg[t1], src);
                  wf4[c] = __uint_as_float(hi ? w1 : w0);
                  const uint32_t pix = static_cast<uint32_t>(hi ? g1 : g0);
                  xv[c] = lane_valid ? ptx::ld_nc_v4(psrc + pix * row_bytes) : make_uint4(0, 0, 0, 0);
                }
                out[r].x = i8_mix_word(wf4, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                out[r].y = i8_mix_word(wf4, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                out[r].z = i8_mix_word(wf4, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                out[r].w = i8_mix_word(wf4, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                if (!lane_valid) out[r] = make_uint4(0, 0, 0, 0);
              }
              const bool got =
                  wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
              if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
              const uint32_t a_s = a_base + s * args.a_stage_bytes;
#pragma unroll
              for (int r = 0; r < R; ++r) ptx::st_shared_v4(a_s + dst_off[r], out[r]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(full_a + 8 * s);
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          } else if (KT > 0 && PREC != PREC_F32 && !args.use_win && (!kPacked || gpacked)) {
            // No window (3x3): every corner is a 16-byte global load of the channels-last x.
            // Straight-line per tap from the cached items (fp16: one shuffle of weight | pixel
            // per corner; int8 / precise fp16: weight and pixel shuffled separately), 32-bit
            // offsets inside the image, lanes past the group's channels predicated off (zeros).
            const uint32_t row_bytes = static_cast<uint32_t>(args.C) * EB;
#pragma unroll
            for (int tt = 0; tt < kCache; ++tt) {
              uint4 out[R];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                uint32_t wv[4];
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int src = grp | (r * 4 + c);
                  wv[c] = __shfl_sync(0xffffffffu, cw[tt], src);
                  const uint32_t pix = kPacked ? (wv[c] >> 16)
                                               : static_cast<uint32_t>(__shfl_sync(0xffffffffu, cg[tt], src));
                  xv[c] = cvalid ? ptx::ld_nc_v4(gsrc + pix * row_bytes) : make_uint4(0, 0, 0, 0);
                }
                if (kPacked) {
                  const __half2 w0 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[0])));
                  const __half2 w1 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[1])));
                  const __half2 w2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[2])));
                  const __half2 w3 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[3])));
                  out[r].x = f16_mix_h2(w0, w1, w2, w3, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[r].y = f16_mix_h2(w0, w1, w2, w3, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[r].z = f16_mix_h2(w0, w1, w2, w3, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[r].w = f16_mix_h2(w0, w1, w2, w3, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                } else {
                  const float wf4[4] = {__uint_as_float(wv[0]), __uint_as_float(wv[1]),
                                        __uint_as_float(wv[2]), __uint_as_float(wv[3])};
                  if (PREC == PREC_I8) {
                    out[r].x = i8_mix_word(wf4, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                    out[r].y = i8_mix_word(wf4, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                    out[r].z = i8_mix_word(wf4, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                    out[r].w = i8_mix_word(wf4, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                  } else {
                    out[r].x = f16_mix_precise(wf4, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                    out[r].y = f16_mix_precise(wf4, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                    out[r].z = f16_mix_precise(wf4, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                    out[r].w = f16_mix_precise(wf4, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                  }
                  if (!cvalid) out[r] = make_uint4(0, 0, 0, 0);
                }
              }
              const bool got =
                  wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
              if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
              const uint32_t a_s = a_base + s * args.a_stage_bytes;
#pragma unroll
              for (int r = 0; r < R; ++r) ptx::st_shared_v4(a_s + dst_off[r], out[r]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(full_a + 8 * s);
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          } else {
            // General path (any tap count, corners outside the window, partial chunks, int8,
            // fp32 and precise fp16). For 3x3 kernels the items come from the per-(tile, group)
            // cache computed above (no geometry load in the K-block loop: a warp's K-block waits
            // on one round trip, its corner loads); otherwise they are recomputed per K-block.
            auto general_kblock = [&](uint32_t myw, int myg) -> bool {
              uint32_t wv[R][4];
              int loc[R][4];  // >= 0: window byte offset; < 0: global pixel -loc - 1
#pragma unroll
              for (int r = 0; r < R; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int src = grp | (r * 4 + c);
                  const uint32_t v = __shfl_sync(0xffffffffu, myw, src);
                  const int gp = __shfl_sync(0xffffffffu, myg, src);
                  if (kPacked) {
                    wv[r][c] = v;
                    loc[r][c] = (KT > 0 && gpacked) ? -static_cast<int>(v >> 16) - 1
                                : (v >> 16) != kNoWin ? static_cast<int>(v >> 16) : -gp - 1;
                  } else {
                    wv[r][c] = v;
                    loc[r][c] = gp < 0 ? (-gp - 1) * kRowBytes : -gp - 1;
                  }
                }
              // loads and mix before the stage is free; stores after
              uint4 outs[R], outs_lo[R];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int e = loc[r][c];
                  if (!cvalid) {
                    xv[c] = make_uint4(0, 0, 0, 0);
                  } else if (e >= 0) {
                    xv[c] = ptx::ld_shared_v4(win + e);
                  } else {
                    xv[c] = ptx::ld_nc_v4(gsrc + static_cast<size_t>(-e - 1) * args.C * EB);
                  }
                }
                uint4 out = make_uint4(0, 0, 0, 0), out_lo = make_uint4(0, 0, 0, 0);
                if (cvalid) {
                  const uint4& x0 = xv[0];
                  const uint4& x1 = xv[1];
                  const uint4& x2 = xv[2];
                  const uint4& x3 = xv[3];
                  if (kPacked) {
                    const __half2 w0 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[r][0])));
                    const __half2 w1 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[r][1])));
                    const __half2 w2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[r][2])));
                    const __half2 w3 = __half2half2(__ushort_as_half(static_cast<unsigned short>(wv[r][3])));
                    out.x = f16_mix_h2(w0, w1, w2, w3, x0.x, x1.x, x2.x, x3.x);
                    out.y = f16_mix_h2(w0, w1, w2, w3, x0.y, x1.y, x2.y, x3.y);
                    out.z = f16_mix_h2(w0, w1, w2, w3, x0.z, x1.z, x2.z, x3.z);
                    out.w = f16_mix_h2(w0, w1, w2, w3, x0.w, x1.w, x2.w, x3.w);
                  } else {
                    const float wf4[4] = {__uint_as_float(wv[r][0]), __uint_as_float(wv[r][1]),
                                          __uint_as_float(wv[r][2]), __uint_as_float(wv[r][3])};
                    if (PREC == PREC_F16) {
                      out.x = f16_mix_precise(wf4, x0.x, x1.x, x2.x, x3.x);
                      out.y = f16_mix_precise(wf4, x0.y, x1.y, x2.y, x3.y);
                      out.z = f16_mix_precise(wf4, x0.z, x1.z, x2.z, x3.z);
                      out.w = f16_mix_precise(wf4, x0.w, x1.w, x2.w, x3.w);
                    } else if (PREC == PREC_I8) {
                      out.x = i8_mix_word(wf4, x0.x, x1.x, x2.x, x3.x);
                      out.y = i8_mix_word(wf4, x0.y, x1.y, x2.y, x3.y);
                      out.z = i8_mix_word(wf4, x0.z, x1.z, x2.z, x3.z);
                      out.w = i8_mix_word(wf4, x0.w, x1.w, x2.w, x3.w);
                    } else {
                      f32_mix(wf4, x0, x1, x2, x3, out, out_lo);
                    }
                  }
                }
                outs[r] = out;
                outs_lo[r] = out_lo;
              }
              const bool got =
                  wait_bar<kSuspend>(empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
              if (!__all_sync(0xffffffffu, got)) return false;
              const uint32_t a_s = a_base + s * args.a_stage_bytes;
#pragma unroll
              for (int r = 0; r < R; ++r) {
                ptx::st_shared_v4(a_s + dst_off[r], outs[r]);
                if (PREC == PREC_F32) ptx::st_shared_v4(a_s + dst_off[r] + kATileBytes, outs_lo[r]);
              }
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(full_a + 8 * s);
              if (++s == S) { s = 0; ph ^= 1u; }
              return true;
            };
            if constexpr (KT > 0) {
#pragma unroll
              for (int tt = 0; tt < kCache; ++tt) {
                ok = general_kblock(cw[tt], cg[tt]);
                if (!ok) break;
              }
            } else {
              for (int t = 0; t < T && ok; ++t) {
                uint32_t myw;
                int myg;
                item(g, t, myw, myg);
                ok = general_kblock(myw, myg);
              }
            }
          }
          if (!ok) break;
          if (args.use_win) {
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(win_empty + 8 * b);
            bool iok = true;
            if (issuer) iok = issue_window(cbi + 2);
            if (!__all_sync(0xffffffffu, iok)) { ok = false; break; }
          }
          ++cbi;
        }
      }
    }
    // Window loads still in flight (only after an abort) must land before the CTA exits.
    if (issuer) {
      for (int q = issued - 2 < 0 ? 0 : issued - 2; q < issued; ++q)
        wait_bar(win_full + 8 * (q & 1), static_cast<uint32_t>(q >> 1) & 1u, wc,
                 DCNV2_DEVERR_TIMEOUT_DRAIN);
    }
  }

  ptx::tc_fence_before();
  // A pair stays resident until both CTAs are done: the leader's MMAs read rank 1's shared memory
  // and rank 1's epilogue arrives on the leader's barriers.
  if (PAIR) ptx::cluster_sync();
  else __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();  // lane 0 ran the MMA loop alone; reconverge for the .sync.aligned dealloc
    ptx::tc_fence_after();
    if (PAIR) ptx::tmem_dealloc_pair(tmem_base, args.tmem_cols);
    else ptx::tmem_dealloc(tmem_base, args.tmem_cols);
  }
}

// ------------------------------------------------------------------ pre-pass: NCHW -> NHWC
// One 16-byte vector moves V = 16/sizeof(T) elements; a tile is TILE = 8*V channels by TILE
// pixels (128-byte rows both ways: 64x64 fp16, 128x128 int8, 32x32 fp32). Rows of the shared
// tile are padded by 4 bytes so that the column reads of the store phase spread over banks.
template <typename T>
__device__ __forceinline__ void transpose_tile(const T* __restrict__ x, T* __restrict__ xt, int C,
                                               int HW, int bx, int by, int n) {
  constexpr int V = 16 / sizeof(T);
  constexpr int TILE = 8 * V;
  constexpr int PAD = 4 / sizeof(T);
  __shared__ T tile[TILE][TILE + PAD];
  const int c0 = by * TILE, p0 = bx * TILE;
  const T* xs = x + static_cast<size_t>(n) * C * HW;
  T* xd = xt + static_cast<size_t>(n) * C * HW;
  const bool vec_in = (HW % V) == 0 && (p0 + TILE) <= HW &&
                      (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  for (int idx = threadIdx.x; idx < TILE * 8; idx += 256) {
    const int i = idx >> 3, q = idx & 7;  // channel row i, 16-byte chunk q of pixels
    const int c = c0 + i;
    if (c < C && vec_in) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(xs + static_cast<size_t>(c) * HW + p0) + q);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < V; ++k) tile[i][q * V + k] = e[k];
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int p = p0 + q * V + k;
        tile[i][q * V + k] = (c < C && p < HW) ? xs[static_cast<size_t>(c) * HW + p] : T(0);
      }
    }
  }
  __syncthreads();
  const bool vec_out = (C % V) == 0 && (c0 + TILE) <= C &&
                       (reinterpret_cast<uintptr_t>(xt) & 15u) == 0;
  for (int idx = threadIdx.x; idx < TILE * 8; idx += 256) {
    const int i = idx >> 3, q = idx & 7;  // pixel row i, 16-byte chunk q of channels
    const int p = p0 + i;
    if (p >= HW) continue;
    if (vec_out) {
      uint4 v;
      T* e = reinterpret_cast<T*>(&v);
#pragma unroll
      for (int k = 0; k < V; ++k) e[k] = tile[q * V + k][i];
      reinterpret_cast<uint4*>(xd + static_cast<size_t>(p) * C + c0)[q] = v;
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int c = c0 + q * V + k;
        if (c < C) xd[static_cast<size_t>(p) * C + c] = tile[q * V + k][i];
      }
    }
  }
}
template <typename T>
__global__ void __launch_bounds__(256) nchw_to_nhwc_kernel(const T* __restrict__ x,
                                                           T* __restrict__ xt, int C, int HW) {
  transpose_tile<T>(x, xt, C, HW, blockIdx.x, blockIdx.y, blockIdx.z);
}

// int8 NCHW -> NHWC for C % 128 == 0 and H*W % 128 == 0 (16-byte aligned pointers): a tile of 128
// channels x 128 pixels. Channel c of the tile sits in shared row (c % 16) * 8 + c / 16 (rows of
// 36 words), so that the 8 channel groups a warp reads at once fall in different bank groups.
// Each thread turns 16 words (16 channels x 4 pixels) into 4 pixels x 16 channels with byte
// permutes (4x4 byte transposes) and writes four 16-byte vectors; the 8 threads of one pixel
// write its 128 channels contiguously.
__device__ __forceinline__ void transpose_i8_tile(const int8_t* __restrict__ x,
                                                  int8_t* __restrict__ xt, int C, int HW, int bx,
                                                  int by, int n) {
  constexpr int kRowWords = 36;
  __shared__ __align__(16) uint32_t tile[128 * kRowWords];
  const int c0 = by * 128, p0 = bx * 128;
  const int8_t* xs = x + static_cast<size_t>(n) * C * HW;
  int8_t* xd = xt + static_cast<size_t>(n) * C * HW;
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (t >> 3) + 32 * i, q = t & 7;  // channel of the tile, 16-pixel chunk
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xs + static_cast<size_t>(c0 + c) * HW + p0) + q);
    const int row = (c & 15) * 8 + (c >> 4);
    *reinterpret_cast<uint4*>(&tile[row * kRowWords + 4 * q]) = v;
  }
  __syncthreads();
  const int cg = t & 7, pg = t >> 3;  // channels 16*cg.., pixels 4*pg..
  uint32_t o[4][4];                   // o[pixel j][word m] = channels 16cg+4m..+3 of pixel 4pg+j
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = tile[((4 * m + k) * 8 + cg) * kRowWords + pg];
    const uint32_t t0 = __byte_perm(w[0], w[1], 0x5140), t1 = __byte_perm(w[0], w[1], 0x7362);
    const uint32_t t2 = __byte_perm(w[2], w[3], 0x5140), t3 = __byte_perm(w[2], w[3], 0x7362);
    o[0][m] = __byte_perm(t0, t2, 0x5410);
    o[1][m] = __byte_perm(t0, t2, 0x7632);
    o[2][m] = __byte_perm(t1, t3, 0x5410);
    o[3][m] = __byte_perm(t1, t3, 0x7632);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(xd + static_cast<size_t>(p0 + 4 * pg + j) * C + c0 + 16 * cg) =
        make_uint4(o[j][0], o[j][1], o[j][2], o[j][3]);
}

// fp16 NCHW -> NHWC for C % 64 == 0 and H*W % 128 == 0 (16-byte aligned pointers): a tile of 64
// channels x 128 pixels. A shared word holds two pixels of one channel; channel c of the tile sits
// in shared row (c % 8) * 8 + c / 8 (rows of 68 words), so the 8 channel groups a warp reads at
// once fall in different bank groups. Each thread turns 8 words (8 channels x 2 pixels) into
// 2 pixels x 8 channels with byte permutes and writes two 16-byte vectors; the 8 threads of one
// pixel write its 64 channels contiguously.
__device__ __forceinline__ void transpose_f16_tile(const __half* __restrict__ x,
                                                   __half* __restrict__ xt, int C, int HW, int bx,
                                                   int by, int n) {
  constexpr int kRowWords = 68;
  __shared__ __align__(16) uint32_t tile[64 * kRowWords];
  const int c0 = by * 64, p0 = bx * 128;
  const __half* xs = x + static_cast<size_t>(n) * C * HW;
  __half* xd = xt + static_cast<size_t>(n) * C * HW;
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (t >> 4) + 16 * i, q = t & 15;  // channel of the tile, 8-pixel chunk
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xs + static_cast<size_t>(c0 + c) * HW + p0) + q);
    const int row = (c & 7) * 8 + (c >> 3);
    *reinterpret_cast<uint4*>(&tile[row * kRowWords + 4 * q]) = v;
  }
  __syncthreads();
  const int cg = t & 7;  // channels 8*cg .. 8*cg+7
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int pp = (t >> 3) + 32 * r;  // pixel pair: pixels 2*pp, 2*pp+1
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = tile[(k * 8 + cg) * kRowWords + pp];
    uint32_t lo[4], hi[4];  // pixel 2pp (low halves) and 2pp+1 (high halves), channel pairs
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      lo[m] = __byte_perm(w[2 * m], w[2 * m + 1], 0x5410);
      hi[m] = __byte_perm(w[2 * m], w[2 * m + 1], 0x7632);
    }
    __half* dst = xd + static_cast<size_t>(p0 + 2 * pp) * C + c0 + 8 * cg;
    *reinterpret_cast<uint4*>(dst) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(dst + C) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
}

// ------------------------------------------------------------------ pre-pass: weight pack
// Writes, for every (cout chunk, K-block), the B operand tile exactly as it must sit in shared
// memory: row o (output channel), 16-byte chunk jc at chunk jc ^ (o % 8) of the 128-byte row.
// K-block kb = (g*CBg + cbg)*T + t holds channels g*Cg + cbg*KC + [0, KC) of tap t.
// Also clears the device error word for the fused kernel that follows.
template <int PREC>
__device__ __forceinline__ void pack_weights_body(const void* __restrict__ w,
                                                  uint8_t* __restrict__ wpack, int* err, int O,
                                                  int C, int T, int Cg, int CBg, int numKB,
                                                  int nrows, int cchunks, int half_mma,
                                                  int tap_pairs, int blk, int nblk) {
  using TR = PrecTraits<PREC>;
  constexpr int EPC = TR::kChunkElems, KC = TR::kBlockElems;
  if (blk == 0 && threadIdx.x == 0) *err = 0;
  const size_t total = static_cast<size_t>(cchunks) * numKB * nrows * 8;
  for (size_t idx = blk * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(nblk) * blockDim.x) {
    const int jc = static_cast<int>(idx & 7);
    const int row = static_cast<int>((idx >> 3) % nrows);
    const size_t blk = (idx >> 3) / nrows;  // cc * numKB + kb
    const int kb = static_cast<int>(blk % numKB);
    const int cc = static_cast<int>(blk / numKB);
    // K order (group, channel block, tap); with tap_pairs (int8, 64-channel groups, CBg = 1)
    // K-block (group, i) holds tap 2i in chunks 0-3 and tap 2i+1 in chunks 4-7
    const int npairs = (T + 1) / 2;
    const int t = tap_pairs ? 2 * (kb % npairs) + (jc >> 2) : kb % T;
    const int cbg = tap_pairs ? 0 : (kb / T) % CBg;
    const int g = tap_pairs ? kb / npairs : kb / (CBg * T);
    const int o = cc * nrows + row;
    const size_t tile_base = blk * TR::kNumBTiles * nrows * kRowBytes;
    // CTA pair (half_mma = n_mma / 2 > 0): rows [sub*n_mma + rk*half_mma, +half_mma) go to CTA
    // rk's half of the K-block, sub-MMA blocks consecutive. half_mma is a multiple of 8, so the
    // swizzle phase (row % 8) is unchanged.
    int srow = row;
    if (half_mma > 0) {
      const int sub = row / (2 * half_mma), r = row - sub * 2 * half_mma;
      const int rk = r / half_mma;
      srow = rk * (nrows / 2) + sub * half_mma + (r - rk * half_mma);
    }
    const size_t dst = tile_base + static_cast<size_t>(srow) * kRowBytes + ((jc ^ (srow & 7)) << 4);
    uint4 hi = make_uint4(0, 0, 0, 0), lo = make_uint4(0, 0, 0, 0);
    uint8_t* hb = reinterpret_cast<uint8_t*>(&hi);
    uint8_t* lb = reinterpret_cast<uint8_t*>(&lo);
#pragma unroll
    for (int e = 0; e < EPC; ++e) {
      const int cig = tap_pairs ? (jc & 3) * EPC + e : cbg * KC + jc * EPC + e;
      if (o < O && cig < Cg && t < T) {
        const size_t src = (static_cast<size_t>(o) * C + g * Cg + cig) * T + t;
        if (PREC == PREC_F16) {
          reinterpret_cast<__half*>(hb)[e] = reinterpret_cast<const __half*>(w)[src];
        } else if (PREC == PREC_I8) {
          reinterpret_cast<int8_t*>(hb)[e] = reinterpret_cast<const int8_t*>(w)[src];
        } else {
          const float v = reinterpret_cast<const float*>(w)[src];
          const uint32_t h = ptx::cvt_rna_tf32(v);
          reinterpret_cast<uint32_t*>(hb)[e] = h;
          reinterpret_cast<uint32_t*>(lb)[e] = ptx::cvt_rna_tf32(v - __uint_as_float(h));
        }
      }
    }
    *reinterpret_cast<uint4*>(wpack + dst) = hi;
    if (TR::kNumBTiles == 2)
      *reinterpret_cast<uint4*>(wpack + dst + static_cast<size_t>(nrows) * kRowBytes) = lo;
  }
}
template <int PREC>
__global__ void __launch_bounds__(256) pack_weights_kernel(const void* __restrict__ w,
                                                           uint8_t* __restrict__ wpack,
                                                           int* err, int O, int C, int T,
                                                           int Cg, int CBg, int numKB,
                                                           int nrows, int cchunks, int half_mma,
                                                           int tap_pairs) {
  pack_weights_body<PREC>(w, wpack, err, O, C, T, Cg, CBg, numKB, nrows, cchunks, half_mma,
                          tap_pairs, blockIdx.x, gridDim.x);
}

// ------------------------------------------------------------------ the two pre-passes, one launch
// Blocks [0, tr_blocks) transpose x to channels-last (tiled kernels where channel and pixel
// counts allow, the generic tile otherwise), the remaining blocks pack the weights into B tiles
// (and clear the error word). The two are independent, so the packing's latency hides under the
// transpose instead of adding a launch after it.
struct PrepassArgs {
  const void* x;
  void* xt;
  int C, HW, tiled;            // tiled: the fp16 / int8 tiled transpose
  int tiles_x, tiles_y, tr_blocks;
  const void* w;
  uint8_t* wpack;
  int* err;
  int O, T, Cg, CBg, numKB, nrows, cchunks, half_mma, tap_pairs;
};

template <int PREC>
__global__ void __launch_bounds__(256) prepass_kernel(const PrepassArgs a) {
  using XT = typename PrecTraits<PREC>::X;
  // the main kernel (launched with programmatic stream serialization) may come up on SMs this
  // grid leaves free and run its setup; it waits for this grid's completion before reading
  ptx::griddep_launch_dependents();
  const int b = static_cast<int>(blockIdx.x);
  if (b < a.tr_blocks) {
    const int bx = b % a.tiles_x, r = b / a.tiles_x;
    const int by = r % a.tiles_y, n = r / a.tiles_y;
    if constexpr (PREC == PREC_F16) {
      if (a.tiled) {
        transpose_f16_tile(static_cast<const __half*>(a.x), static_cast<__half*>(a.xt), a.C, a.HW,
                           bx, by, n);
        return;
      }
    } else if constexpr (PREC == PREC_I8) {
      if (a.tiled) {
        transpose_i8_tile(static_cast<const int8_t*>(a.x), static_cast<int8_t*>(a.xt), a.C, a.HW,
                          bx, by, n);
        return;
      }
    }
    transpose_tile<XT>(static_cast<const XT*>(a.x), static_cast<XT*>(a.xt), a.C, a.HW, bx, by, n);
  } else {
    pack_weights_body<PREC>(a.w, a.wpack, a.err, a.O, a.C, a.T, a.Cg, a.CBg, a.numKB, a.nrows,
                            a.cchunks, a.half_mma, a.tap_pairs, b - a.tr_blocks,
                            static_cast<int>(gridDim.x) - a.tr_blocks);
  }
}

// ------------------------------------------------------------------ fp32-exact fused kernel
// The tensor-core accumulator does not add with fp32 round-to-nearest at every step, and over
// the ~900 accumulation steps of a 3xTF32 product at C*K*K = 2304 its error reaches ~5e-5
// relative. This kernel is the fp32-exact path: the same fused structure (samples go straight
// to shared memory, K ordered (group, tap, 32-channel block), no column matrix in HBM), with the
// GEMM on CUDA cores in fp32 FMA. CTA tile: 64 output pixels x 128 output channels, computed by
// two groups of 256 threads that split the K-blocks in halves (each thread accumulates 4 pixels x
// 8 channels of its half; double-buffered shared-memory stages per group); the second group's
// sums are added to the first's at the end, so every output is (first half) + (second half) +
// bias whatever the batch. Two groups give 16 warps per SM where one image leaves 128 CTAs for
// 148 SMs.
constexpr int kXPx = 64, kXCo = 128, kXK = 32, kXThreads = 256, kXGroups = 2;
// dynamic shared memory: per group A [2][kXK][kXPx] and B [2][kXK][kXCo] floats
constexpr int kXGroupFloats = 2 * kXK * kXPx + 2 * kXK * kXCo;
constexpr size_t kXSmemBytes = size_t(kXGroups) * kXGroupFloats * sizeof(float);

struct ExactArgs {
  const float* x_nhwc;   // [N][H][W][C]
  const float* offset;   // [N][dg*2*T][Ho][Wo]
  const float* mask;     // [N][dg*T][Ho][Wo]
  const float* wplain;   // [ctiles][numKB][32][128] (k-major rows of 128 output channels)
  const float* bias;
  float* y;
  int N, C, H, W, O, Ho, Wo, P, K, T, stride, pad, dil, dg, Cg, CBg, numKB;
  int ptiles, ctiles;
};

__global__ void __launch_bounds__(kXThreads * kXGroups, 1) dcnv2_f32_exact_kernel(const ExactArgs a) {
  extern __shared__ __align__(16) float xsm[];
  // launched with programmatic stream serialization: the pre-pass's outputs are read from here
  ptx::griddep_wait();
  const int grp = threadIdx.x / kXThreads;  // K half
  const int tid = threadIdx.x - grp * kXThreads;
  float (*As)[kXK][kXPx] = reinterpret_cast<float (*)[kXK][kXPx]>(xsm + grp * kXGroupFloats);
  float (*Bs)[kXK][kXCo] =
      reinterpret_cast<float (*)[kXK][kXCo]>(xsm + grp * kXGroupFloats + 2 * kXK * kXPx);
  const int half = (a.numKB + 1) / 2;
  const int kb_begin = grp == 0 ? 0 : half, kb_end = grp == 0 ? half : a.numKB;
  // the two groups synchronise separately (their K ranges may differ in length)
  auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(kXThreads)); };
  const int ct = blockIdx.x % a.ctiles;
  const int pt = (blockIdx.x / a.ctiles) % a.ptiles;
  const int img = blockIdx.x / (a.ctiles * a.ptiles);
  // sampler role: pixel sp, channels sq*8 .. sq*8+7 of the 32-channel block
  const int sp = tid & (kXPx - 1), sq = tid >> 6;
  const int p = pt * kXPx + sp;
  const bool pvalid = p < a.P;
  const int pc = pvalid ? p : 0;
  const int oh = pc / a.Wo, ow = pc - oh * a.Wo;
  // compute role: pixels ty*4 .. +4, output channels tx*4 .. +4 and 64 + tx*4 .. +4 (the two
  // float4 reads of a half-warp cover 256 contiguous bytes: no bank conflicts)
  const int ty = tid >> 4, tx = tid & 15;
  const float* ximg = a.x_nhwc + static_cast<size_t>(img) * a.H * a.W * a.C;
  const float* wct = a.wplain + static_cast<size_t>(ct) * a.numKB * kXK * kXCo;

  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  // prefetched state of the next K-block
  float4 bq[4];
  float4 xc[4][2];
  float gw[4] = {0.f, 0.f, 0.f, 0.f};
  int gof[4] = {0, 0, 0, 0};
  bool cval[2];

  auto prefetch = [&](int kb) {
    const int cbg = kb % a.CBg;
    const int t = (kb / a.CBg) % a.T;
    const int g = kb / (a.CBg * a.T);
    if (cbg == 0 || kb == kb_begin) {  // new (group, tap): new sampling geometry
      const int ki = t / a.K, kj = t - ki * a.K;
      float dh = 0.f, dw = 0.f, m = 0.f;
      if (pvalid) {
        const size_t go = (static_cast<size_t>(img) * a.dg + g) * 2 * a.T + 2 * t;
        const size_t gm = (static_cast<size_t>(img) * a.dg + g) * a.T + t;
        dh = __ldg(a.offset + go * a.P + p);
        dw = __ldg(a.offset + (go + 1) * a.P + p);
        m = __ldg(a.mask + gm * a.P + p);
      }
      FusedArgs ga;
      ga.H = a.H; ga.W = a.W; ga.C = a.C;
      const Geom gm = make_geom(ga, pvalid, oh * a.stride - a.pad + ki * a.dil,
                                ow * a.stride - a.pad + kj * a.dil, dh, dw, m);
#pragma unroll
      for (int c = 0; c < 4; ++c) { gw[c] = gm.a[c]; gof[c] = gm.off[c]; }
    }
    const int cig = cbg * kXK + sq * 8;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      cval[h] = (cig + 4 * h) < a.Cg;
      const int cb = g * a.Cg + cig + 4 * h;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        xc[c][h] = cval[h] ? __ldg(reinterpret_cast<const float4*>(ximg + gof[c] + cb))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float4* bsrc = reinterpret_cast<const float4*>(wct + static_cast<size_t>(kb) * kXK * kXCo);
#pragma unroll
    for (int i = 0; i < 4; ++i) bq[i] = __ldg(bsrc + tid + i * kXThreads);
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float* x0 = &xc[0][h].x; const float* x1 = &xc[1][h].x;
      const float* x2 = &xc[2][h].x; const float* x3 = &xc[3][h].x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = __fmul_rn(gw[0], x0[e]);
        v = __fmaf_rn(gw[1], x1[e], v);
        v = __fmaf_rn(gw[2], x2[e], v);
        v = __fmaf_rn(gw[3], x3[e], v);
        As[buf][sq * 8 + 4 * h + e][sp] = cval[h] ? v : 0.f;
      }
    }
    float4* bd = reinterpret_cast<float4*>(&Bs[buf][0][0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) bd[tid + i * kXThreads] = bq[i];
  };

  if (kb_begin < kb_end) {
    prefetch(kb_begin);
    store(0);
  }
  group_sync();
  for (int kb = kb_begin; kb < kb_end; ++kb) {
    const int buf = (kb - kb_begin) & 1;
    const bool more = kb + 1 < kb_end;
    if (more) prefetch(kb + 1);
#pragma unroll 8
    for (int k = 0; k < kXK; ++k) {
      const float4 av = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][kXCo / 2 + tx * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float br[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(ar[i], br[j], acc[i][j]);
    }
    if (more) store(buf ^ 1);
    group_sync();
  }
  // the second half's sums, through shared memory ([32 values][256 threads]: conflict-free)
  float* red = xsm + kXGroupFloats;
  if (grp == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[(i * 8 + j) * kXThreads + tid] = acc[i][j];
  }
  __syncthreads();
  if (grp == 1) return;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = __fadd_rn(acc[i][j], red[(i * 8 + j) * kXThreads + tid]);
  float* yimg = a.y + static_cast<size_t>(img) * a.O * a.P;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int o = ct * kXCo + (j < 4 ? tx * 4 + j : kXCo / 2 + tx * 4 + (j - 4));
    if (o >= a.O) continue;
    const float bo = a.bias ? __ldg(a.bias + o) : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pp = pt * kXPx + ty * 4 + i;
      if (pp < a.P) yimg[static_cast<size_t>(o) * a.P + pp] = acc[i][j] + bo;
    }
  }
}

// Weights for the fp32-exact kernel: [ctile][kb][k][128 co], zero padded.
__device__ __forceinline__ void pack_weights_plain_body(const float* __restrict__ w,
                                                        float* __restrict__ wp, int* err, int O,
                                                        int C, int T, int Cg, int CBg, int numKB,
                                                        int ctiles, int blk, int nblk) {
  if (blk == 0 && threadIdx.x == 0) *err = 0;
  const size_t total = static_cast<size_t>(ctiles) * numKB * kXK * kXCo;
  for (size_t idx = blk * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(nblk) * blockDim.x) {
    const int co = static_cast<int>(idx % kXCo);
    const int k = static_cast<int>((idx / kXCo) % kXK);
    const size_t blk = idx / (static_cast<size_t>(kXCo) * kXK);
    const int kb = static_cast<int>(blk % numKB);
    const int ct = static_cast<int>(blk / numKB);
    const int cbg = kb % CBg, t = (kb / CBg) % T, g = kb / (CBg * T);
    const int o = ct * kXCo + co;
    const int cig = cbg * kXK + k;
    float v = 0.f;
    if (o < O && cig < Cg) v = w[(static_cast<size_t>(o) * C + g * Cg + cig) * T + t];
    wp[idx] = v;
  }
}

// The fp32-exact path's two pre-passes in one launch, as prepass_kernel: blocks [0, tr_blocks)
// transpose x to channels-last (32 x 32 tiles), the rest pack the weights k-major.
struct PrepassPlainArgs {
  const float* x;
  float* xt;
  int C, HW, tiles_x, tiles_y, tr_blocks;
  const float* w;
  float* wp;
  int* err;
  int O, T, Cg, CBg, numKB, ctiles;
};

__global__ void __launch_bounds__(256) prepass_plain_kernel(const PrepassPlainArgs a) {
  ptx::griddep_launch_dependents();
  const int b = static_cast<int>(blockIdx.x);
  if (b < a.tr_blocks) {
    const int bx = b % a.tiles_x, r = b / a.tiles_x;
    transpose_tile<float>(a.x, a.xt, a.C, a.HW, bx, r % a.tiles_y, r / a.tiles_y);
  } else {
    pack_weights_plain_body(a.w, a.wp, a.err, a.O, a.C, a.T, a.Cg, a.CBg, a.numKB, a.ctiles,
                            b - a.tr_blocks, static_cast<int>(gridDim.x) - a.tr_blocks);
  }
}

// ------------------------------------------------------------------ CUDA-core fallback
// One thread per output element, any shape (the reference's naive kernel structure,
// src/dcn_kernel.cu:33-65, extended to N, groups and the int8 requantisation). Column values use
// the same geometry and mixing order as the fused kernels; fp16 columns are rounded to fp16, int8
// columns follow the fixed-point rule at i8_mix_fx.
struct SimtArgs {
  const void* x; const void* offset; const void* mask; const void* w; const void* bias; void* y;
  int N, C, H, W, O, Ho, Wo, P, K, T, stride, pad, dil, dg, Cg;
  float scale;
  int i8_rint;  // int8: column = clamp(rint(m * bilinear(x_q)), -127, 127) in fp32 (see below)
};

template <int PREC>
__global__ void __launch_bounds__(256) dcnv2_simt_kernel(const SimtArgs a) {
  using TR = PrecTraits<PREC>;
  using XT = typename TR::X;
  using GT = typename TR::G;
  const size_t total = static_cast<size_t>(a.N) * a.O * a.P;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(idx % a.P);
    const int o = static_cast<int>((idx / a.P) % a.O);
    const int n = static_cast<int>(idx / (static_cast<size_t>(a.P) * a.O));
    const int oh = p / a.Wo, ow = p - (p / a.Wo) * a.Wo;
    const XT* xn = reinterpret_cast<const XT*>(a.x) + static_cast<size_t>(n) * a.C * a.H * a.W;
    const GT* offp = reinterpret_cast<const GT*>(a.offset);
    const GT* maskp = reinterpret_cast<const GT*>(a.mask);
    float facc = 0.f;
    long long iacc = 0;
    for (int g = 0; g < a.dg; ++g) {
      for (int t = 0; t < a.T; ++t) {
        const int ki = t / a.K, kj = t - ki * a.K;
        const size_t goff = (static_cast<size_t>(n) * a.dg + g) * 2 * a.T + 2 * t;
        const size_t gmsk = (static_cast<size_t>(n) * a.dg + g) * a.T + t;
        const float dh = load_geom_value(offp + goff * a.P + p);
        const float dw = load_geom_value(offp + (goff + 1) * a.P + p);
        const float m_raw = load_geom_value(maskp + gmsk * a.P + p);
        const float m = PREC == PREC_I8 ? i8_mask(m_raw) : m_raw;
        const float hf = __fadd_rn(static_cast<float>(oh * a.stride - a.pad + ki * a.dil), dh);
        const float wf = __fadd_rn(static_cast<float>(ow * a.stride - a.pad + kj * a.dil), dw);
        const bool inside = !(hf <= -1.f || hf >= static_cast<float>(a.H) || wf <= -1.f ||
                              wf >= static_cast<float>(a.W));
        float wt[4] = {0.f, 0.f, 0.f, 0.f};
        float area[4] = {0.f, 0.f, 0.f, 0.f};  // corner areas without the mask (int8 rint rule)
        int idx4[4] = {-1, -1, -1, -1};
        if (inside) {
          const float h0f = floorf(hf), w0f = floorf(wf);
          const int h0 = static_cast<int>(h0f), w0 = static_cast<int>(w0f);
          const float lh = __fsub_rn(hf, h0f), lw = __fsub_rn(wf, w0f);
          const float hh = __fsub_rn(1.f, lh), hw = __fsub_rn(1.f, lw);
          area[0] = __fmul_rn(hh, hw); area[1] = __fmul_rn(hh, lw);
          area[2] = __fmul_rn(lh, hw); area[3] = __fmul_rn(lh, lw);
          if (h0 >= 0 && w0 >= 0) { wt[0] = __fmul_rn(m, __fmul_rn(hh, hw)); idx4[0] = h0 * a.W + w0; }
          if (h0 >= 0 && w0 + 1 <= a.W - 1) { wt[1] = __fmul_rn(m, __fmul_rn(hh, lw)); idx4[1] = h0 * a.W + w0 + 1; }
          if (h0 + 1 <= a.H - 1 && w0 >= 0) { wt[2] = __fmul_rn(m, __fmul_rn(lh, hw)); idx4[2] = (h0 + 1) * a.W + w0; }
          if (h0 + 1 <= a.H - 1 && w0 + 1 <= a.W - 1) { wt[3] = __fmul_rn(m, __fmul_rn(lh, lw)); idx4[3] = (h0 + 1) * a.W + w0 + 1; }
        }
        for (int ci = 0; ci < a.Cg; ++ci) {
          const int c = g * a.Cg + ci;
          const XT* plane = xn + static_cast<size_t>(c) * a.H * a.W;
          float xv[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (idx4[k] >= 0) {
              if (PREC == PREC_F16) xv[k] = __half2float(reinterpret_cast<const __half*>(plane)[idx4[k]]);
              else if (PREC == PREC_I8) xv[k] = static_cast<float>(reinterpret_cast<const int8_t*>(plane)[idx4[k]]);
              else xv[k] = reinterpret_cast<const float*>(plane)[idx4[k]];
            } else {
              xv[k] = 0.f;
            }
          }
          float v = __fmul_rn(wt[0], xv[0]);
          v = __fmaf_rn(wt[1], xv[1], v);
          v = __fmaf_rn(wt[2], xv[2], v);
          v = __fmaf_rn(wt[3], xv[3], v);
          const size_t widx = (static_cast<size_t>(o) * a.C + c) * a.T + t;
          if (PREC == PREC_I8) {
            int q;
            if (a.i8_rint) {
              // The reference's fp32 column m * bilinear(x_q) (src/dcn_kernel.cu:19-30, :234),
              // every product and sum rounded as written (corner area * value, left to right,
              // then times the unclamped mask), rounded to nearest even and clamped to +-127.
              float b = __fmul_rn(area[0], xv[0]);
              b = __fadd_rn(b, __fmul_rn(area[1], xv[1]));
              b = __fadd_rn(b, __fmul_rn(area[2], xv[2]));
              b = __fadd_rn(b, __fmul_rn(area[3], xv[3]));
              const float cv = __fmul_rn(m_raw, b);
              q = __float2int_rn(cv);  // NaN -> 0
              q = q < -127 ? -127 : (q > 127 ? 127 : q);
            } else {
              int sum = 32768;  // fixed-point column value (rule at i8_mix_fx)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                sum += static_cast<int>(i8_weight(wt[k])) * static_cast<int>(xv[k]);
              q = sum >> 16;
            }
            iacc += static_cast<long long>(q) * reinterpret_cast<const int8_t*>(a.w)[widx];
          } else if (PREC == PREC_F16) {
            const float cv = __half2float(__float2half_rn(v));
            facc = __fmaf_rn(__half2float(reinterpret_cast<const __half*>(a.w)[widx]), cv, facc);
          } else {
            facc = __fmaf_rn(reinterpret_cast<const float*>(a.w)[widx], v, facc);
          }
        }
      }
    }
    if (PREC == PREC_F16) {
      const float bo = a.bias ? __half2float(reinterpret_cast<const __half*>(a.bias)[o]) : 0.f;
      reinterpret_cast<__half*>(a.y)[idx] = __float2half_rn(facc + bo);
    } else if (PREC == PREC_I8) {
      const float bo = a.bias ? reinterpret_cast<const float*>(a.bias)[o] : 0.f;
      reinterpret_cast<float*>(a.y)[idx] =
          __fmaf_rn(static_cast<float>(iacc), a.scale, bo);
    } else {
      const float bo = a.bias ? reinterpret_cast<const float*>(a.bias)[o] : 0.f;
      reinterpret_cast<float*>(a.y)[idx] = facc + bo;
    }
  }
}

}  // namespace dcnv2
