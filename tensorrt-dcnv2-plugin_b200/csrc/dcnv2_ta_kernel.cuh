// dcnv2_ta_kernel.cuh — fused DCNv2 forward with the sampled A operand in tensor memory.
//
// Same implicit GEMM as dcnv2_fused_kernel (D[128 pixels, O] = A[128 pixels, C*K*K] *
// B[O, C*K*K]^T, K ordered (group, channel block, tap), one TMA window of channels-last x per
// channel block), with one change of data path: the samplers write the bilinear samples of a
// K-block into tensor memory (tcgen05.st) instead of shared memory, and tcgen05.mma reads A from
// there. Per K-block of 128 pixels x 128 bytes this saves the 16 KB shared-memory store of the A
// tile and the tensor core's 16 KB shared-memory read of it, which leaves shared memory to the
// corner reads (64 KB) and the weight tiles. TMEM holds the accumulator (256 columns, so at most
// 256 output channels per tile; wider layers run several output-channel chunks), for fp16 a park
// area of 128 columns (the converted tile, stored to y while the next tile's MMAs run), and a
// ring of A stages of 32 columns (4 for fp16, 8 for int8).
//
// Roles (576 threads; 18 warps leave each thread 96 registers):
//   warp 0       producer: bulk copy of each K-block's pre-swizzled weight tile (B ring, smem)
//   warp 1       MMA issuer (lane 0): tcgen05.mma kind::f16 / kind::i8, A from TMEM, B from smem
//   warps 2-5    epilogue: tcgen05.ld of the accumulator, + bias (x x_scale*w_scale for int8),
//                stores of y (two pixels per store where the layout allows)
//   warps 6-17   samplers: warp w fills TMEM lane quadrant w % 4 (32 pixels, thread = pixel),
//                whole 128-byte rows of the K-blocks of taps t = (w - 6) / 4 (mod 3)
// The x window is stored linearly (128 bytes per pixel, so 16-byte chunk c of any pixel sits in
// bank group c). In the 3x3 fast path (fp16 and int8) lane i reads chunk h ^ (i % 8) at step h:
// the 8 lanes of each 128-bit load phase hit 8 different bank groups whatever the offsets, and a
// register butterfly restores the chunk order before the TMEM store. The x windows are double
// buffered; the sampler warp that is last to finish with a buffer issues the TMA load of the
// window two channel blocks ahead into it (a shared-memory count per buffer), so no sampler
// waits for the others at a channel-block boundary.
#pragma once
#include "dcnv2_kernels.cuh"

namespace dcnv2 {

constexpr uint32_t kTaAccCols = 256;   // accumulator: one 32-bit column per output channel
constexpr uint32_t kTaStageCols = 32;  // one A K-block: 128 bytes of every TMEM lane
constexpr int kTaMaxAStages = 8;       // (512 - 256) / 32
// fp16: the epilogue parks the converted tile (256 fp16 channels of each pixel = 128 columns)
// next to the accumulator and releases the accumulator before it stores y, so the MMAs of the
// next tile wait only for the TMEM-to-TMEM drain; 4 A stages remain.
constexpr uint32_t kTaParkCols = 128;
template <int PREC> struct TaLayout {
  static constexpr bool kPark = PREC == PREC_F16;
  static constexpr uint32_t kACol0 = kTaAccCols + (kPark ? kTaParkCols : 0);
  static constexpr int kAStages = kPark ? 4 : kTaMaxAStages;
};
constexpr uint32_t kTaTmemCols = 512;
constexpr int kTaMaxBStages = 8;
constexpr int kTaTapGroups = 3;        // sampler warps per TMEM lane quadrant
constexpr int kTaSampWarps = 4 * kTaTapGroups;
constexpr int kTaThreads = (kSampWarp0 + kTaSampWarps) * 32;  // 576: 18 warps, 96 registers

struct TaMmaParams {
  uint32_t b_base, b_stage_bytes, tmem_base;
  uint32_t a_full, a_empty, b_full, b_empty, tfull, tempty, drain;
  int SA, SB, num_tiles, tile0, tstep, numKB, n_mma;
  WaitCtx wc;
};

// Single MMA lane (not inlined: its loop keeps its own registers). Per K-block: wait for the A
// stage (TMEM) and the B stage (smem), 4 K-steps of tcgen05.mma, then one commit per ring so
// that each stage is released as soon as the MMAs reading it complete. One accumulator: a tile
// starts after the epilogue has read the previous one; the A ring keeps the samplers busy
// meanwhile.
template <int PREC>
__device__ __noinline__ void ta_mma_issuer(const TaMmaParams mp) {
  const uint32_t m = kTileM;
  const uint32_t idesc = PREC == PREC_F16 ? ptx::make_idesc(1, 0, mp.n_mma, m)
                                          : ptx::make_idesc(2, 1, mp.n_mma, m);
  const uint64_t desc0 = ptx::sw128_kmajor_desc(0);
  const uint32_t a_tm0 = mp.tmem_base + TaLayout<PREC>::kACol0;
  const WaitCtx& wc = mp.wc;
  int sa = 0, sb = 0;
  uint32_t pa = 0, pb = 0, use = 0;
  bool ok = true;
  for (int tile = mp.tile0; tile < mp.num_tiles && ok; tile += mp.tstep) {
    // the accumulator drained: a suspended wait wakes when the phase completes
    if (!wait_bar<kSuspend>(mp.tempty, use ^ 1u, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    ptx::tc_fence_after();
    // `ready`: the barriers of K-block kb were found complete by the look-ahead test made while
    // the previous K-block's MMAs were queued (its latency overlaps tensor work)
    bool ready = false;
    for (int kb = 0; kb < mp.numKB; ++kb) {
      if (!ready) {
        if (!wait_bar(mp.b_full + 8 * sb, pb, wc, DCNV2_DEVERR_TIMEOUT_MMA) ||
            !wait_bar(mp.a_full + 8 * sa, pa, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
      }
      ptx::tc_fence_after();
      const uint32_t at = a_tm0 + static_cast<uint32_t>(sa) * kTaStageCols;
      const uint64_t bd0 = desc0 | (((mp.b_base + sb * mp.b_stage_bytes) >> 4) & 0x3FFFu);
      // next stage indices, and a non-blocking test of its barriers
      const int sa1 = sa + 1 == mp.SA ? 0 : sa + 1, sb1 = sb + 1 == mp.SB ? 0 : sb + 1;
      const uint32_t pa1 = sa + 1 == mp.SA ? pa ^ 1u : pa, pb1 = sb + 1 == mp.SB ? pb ^ 1u : pb;
      uint32_t nxt = 0;
      if (kb + 1 < mp.numKB) {
        nxt = ptx::mbar_test_wait(mp.b_full + 8 * sb1, pb1) &
              ptx::mbar_test_wait(mp.a_full + 8 * sa1, pa1);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // K-step k: 8 TMEM columns of A, 32 bytes further along the B rows
        const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
        if (PREC == PREC_F16) ptx::mma_f16_ta(mp.tmem_base, at + 8 * k, bd0 + 2 * k, idesc, accum);
        else ptx::mma_i8_ta(mp.tmem_base, at + 8 * k, bd0 + 2 * k, idesc, accum);
      }
      ptx::tc_commit(mp.a_empty + 8 * sa);
      ptx::tc_commit(mp.b_empty + 8 * sb);
      sa = sa1; sb = sb1; pa = pa1; pb = pb1;
      ready = nxt != 0;
    }
    if (!ok) break;
    ptx::tc_commit(mp.tfull);
    use ^= 1u;
  }
  ptx::tc_commit(mp.drain);
  wait_bar(mp.drain, 0, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
}

// Bilinear geometry of tap t for one pixel: the four corner weights (mask folded in, zero when a
// corner or the sample centre is outside the image; the rules of bilinear<T>,
// src/dcn_kernel.cu:19-30) and where each corner is read: loc >= 0 is the byte offset, inside
// the window of the corner pixel (chunk h is at loc + 16 h); loc < 0 is -(pixel index in the
// channels-last image) - 1. Operations and their order match make_geom.
__device__ __forceinline__ void ta_tap_geom(const FusedArgs& a, bool valid, int bh, int bw,
                                            float dh, float dw, float m, int row0,
                                            float (&wt)[4], int (&loc)[4]) {
  const float hf = __fadd_rn(static_cast<float>(bh), dh);
  const float wf = __fadd_rn(static_cast<float>(bw), dw);
  const bool inside = valid && !(hf <= -1.f || hf >= static_cast<float>(a.H) || wf <= -1.f ||
                                 wf >= static_cast<float>(a.W));
  const float h0f = floorf(hf), w0f = floorf(wf);
  const int h0 = inside ? static_cast<int>(h0f) : 0;
  const int w0 = inside ? static_cast<int>(w0f) : 0;
  const float lh = __fsub_rn(hf, h0f), lw = __fsub_rn(wf, w0f);
  const float hh = __fsub_rn(1.f, lh), hw = __fsub_rn(1.f, lw);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int dy = c >> 1, dx = c & 1;
    const float fy = dy ? lh : hh, fx = dx ? lw : hw;
    const int hc = h0 + dy, wc = w0 + dx;
    const bool cok = inside && hc >= 0 && hc <= a.H - 1 && wc >= 0 && wc <= a.W - 1;
    wt[c] = cok ? __fmul_rn(m, __fmul_rn(fy, fx)) : 0.f;
    if (a.use_win && (!cok || (hc >= row0 && hc < row0 + a.win_rows))) {
      const int wp = cok ? (hc - row0) * a.W + wc : 0;
      loc[c] = wp * kRowBytes;
    } else {
      loc[c] = -(cok ? hc * a.W + wc : 0) - 1;
    }
  }
}

// Slot h of `o` (words 4h..4h+3) holds chunk h ^ r; afterwards slot c holds chunk c. Three
// conditional exchanges of slots h and h ^ 2^b (b = 0, 1, 2), each when bit b of r is set.
template <int B>
__device__ __forceinline__ void xchg_slots(uint32_t (&o)[32], bool p) {
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    if (h & (1 << B)) continue;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t a = o[4 * h + w], b = o[4 * (h | (1 << B)) + w];
      o[4 * h + w] = p ? b : a;
      o[4 * (h | (1 << B)) + w] = p ? a : b;
    }
  }
}
__device__ __forceinline__ void unrotate_chunks(uint32_t (&o)[32], int r) {
  xchg_slots<0>(o, r & 1);
  xchg_slots<1>(o, r & 2);
  xchg_slots<2>(o, r & 4);
}

template <int PREC, bool PRECISE, int KT>
__global__ void __launch_bounds__(kTaThreads, 1)
    dcnv2_fused_ta_kernel(const FusedArgs args, const __grid_constant__ CUtensorMap tmap_x) {
  using TR = PrecTraits<PREC>;
  using GT = typename TR::G;
  using YT = typename TR::Y;
  static_assert(PREC == PREC_F16 || PREC == PREC_I8, "A in TMEM: fp16 and int8 only");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int SA = args.a_stages, SB = args.b_stages;
  // [2 windows (1 KB aligned) | SB B stages | barriers | bias]
  uint8_t* w_smem = smem;
  uint8_t* b_smem = smem + (args.use_win ? 2 * args.win_stride : 0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_smem + static_cast<size_t>(SB) * args.b_stage_bytes);
  const uint32_t a_full = ptx::smem_addr(bars);   // [SA] sampler warps -> MMA
  const uint32_t a_empty = a_full + 8 * SA;       // [SA] MMA commit -> samplers
  const uint32_t b_full = a_empty + 8 * SA;       // [SB] weight copy landed
  const uint32_t b_empty = b_full + 8 * SB;       // [SB] MMA commit -> producer
  const uint32_t tfull = b_empty + 8 * SB;        // accumulator ready
  const uint32_t tempty = tfull + 8;              // accumulator read by the epilogue(s)
  const uint32_t drain = tempty + 8;
  const uint32_t win_full = drain + 8;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SA + 2 * SB + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [2] sampler warps done with window buffer b, counted over the kernel (the warp that
  // completes a use loads the buffer's next window), and the number of windows issued
  uint32_t* win_done = tmem_slot + 2;
  uint32_t* win_issued = tmem_slot + 4;
  // bias of the (single) output-channel chunk as fp32, after the 512 bytes of barriers
  float* bias_smem = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512);
  const WaitCtx wc{args.timeout_ns, args.err, abort_flag};
  const int tile0 = static_cast<int>(blockIdx.x);
  const int tstep = static_cast<int>(gridDim.x);
  auto pix_base = [&](int pt) { return pt * kTileM; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      ptx::mbar_init(a_full + 8 * s, 4);  // one sampler warp per lane quadrant
      ptx::mbar_init(a_empty + 8 * s, 1);
    }
    for (int s = 0; s < SB; ++s) {
      ptx::mbar_init(b_full + 8 * s, 1);
      ptx::mbar_init(b_empty + 8 * s, 1);
    }
    ptx::mbar_init(tfull, 1);
    ptx::mbar_init(tempty, kNumEpiWarps);
    ptx::mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(win_full + 8 * i, 1);
      win_done[i] = 0;
    }
    *win_issued = 0;
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (args.cchunks == 1) {
    for (int i = threadIdx.x; i < args.n_mma; i += blockDim.x) {
      float bv = 0.f;
      if (args.bias && i < args.O)
        bv = PREC == PREC_F16 ? __half2float(reinterpret_cast<const __half*>(args.bias)[i])
                              : reinterpret_cast<const float*>(args.bias)[i];
      bias_smem[i] = bv;
    }
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), kTaTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
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
      const size_t kb_bytes = static_cast<size_t>(args.b_stage_bytes);
      for (int tile = tile0; tile < args.num_tiles && ok; tile += tstep) {
        int img, pt, cc;
        decode_tile(args, tile, img, pt, cc);
        const uint8_t* src = args.wpack + static_cast<size_t>(cc) * args.numKB * kb_bytes;
        for (int kb = 0; kb < args.numKB; ++kb, ++it) {
          if (!wait_bar<kSuspend>(b_empty + 8 * s, ph ^ 1, wc, DCNV2_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(b_full + 8 * s, args.b_stage_bytes);
          ptx::bulk_copy_g2s(b_base + s * args.b_stage_bytes,
                             src + static_cast<size_t>(kb) * kb_bytes, args.b_stage_bytes,
                             b_full + 8 * s);
          if (++s == SB) { s = 0; ph ^= 1u; }
        }
      }
      // copies still in flight (at most the last one per stage) land before the CTA exits
      const int outstanding = it < SB ? it : SB;
      for (int j = 0; j < outstanding; ++j) {
        const int idx = it - 1 - j;
        wait_bar(b_full + 8 * (idx % SB), (idx / SB) & 1, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      TaMmaParams mp;
      mp.b_base = ptx::smem_addr(b_smem);
      mp.b_stage_bytes = args.b_stage_bytes;
      mp.tmem_base = tmem_base;
      mp.a_full = a_full; mp.a_empty = a_empty; mp.b_full = b_full; mp.b_empty = b_empty;
      mp.tfull = tfull; mp.tempty = tempty; mp.drain = drain;
      mp.SA = SA; mp.SB = SB; mp.num_tiles = args.num_tiles; mp.tile0 = tile0;
      mp.tstep = tstep; mp.numKB = args.numKB; mp.n_mma = args.n_mma;
      mp.wc = wc;
      ta_mma_issuer<PREC>(mp);
    }
  } else if (warp < kSampWarp0) {
    // ------------------------------------------------------------ epilogue
    // Per 16 accumulator columns: tcgen05.ld (the next block's load overlaps this block's
    // stores), + bias from shared memory (staged at kernel start), convert, store: int8 through
    // epilogue_block; fp16 parks the converted tile in TMEM first (below).
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const bool paired = (args.P % 2) == 0 &&
                        (reinterpret_cast<uintptr_t>(args.y) % (2 * sizeof(YT))) == 0;
    const bool staged = args.cchunks == 1;
    const int odd = lane & 1;
    int tl = 0;
    for (int tile = tile0; tile < args.num_tiles; tile += tstep, ++tl) {
      const bool got = wait_bar<kSuspend, false>(tfull, static_cast<uint32_t>(tl) & 1u, wc,
                                                 DCNV2_DEVERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      ptx::tc_fence_after();
      int img, pt, cc;
      decode_tile(args, tile, img, pt, cc);
      const int p = pix_base(pt) + q * 32 + lane;
      const int pe = p - odd;  // first pixel of this lane's pair
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      const int o_chunk = cc * args.n_mma;
      const int ncols = args.O - o_chunk < args.n_mma ? args.O - o_chunk : args.n_mma;
      YT* yimg = reinterpret_cast<YT*>(args.y) + static_cast<size_t>(img) * args.O * args.P;
      auto release = [&]() {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(tempty);
        }
      };
      uint32_t ra[16], rb[16];
      if constexpr (TaLayout<PREC>::kPark) {
        // 1) accumulator + bias -> fp16 pairs in the park columns, then release the accumulator
        const uint32_t park = taddr + kTaAccCols;
        auto drain = [&](uint32_t (&r)[16], int col) {
          uint32_t h[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 b2 = staged ? *reinterpret_cast<const float2*>(bias_smem + col + 2 * i)
                                     : make_float2(0.f, 0.f);
            float b0 = b2.x, b1 = b2.y;
            if (!staged && args.bias) {
              const int o = o_chunk + col + 2 * i;
              const __half* bp = reinterpret_cast<const __half*>(args.bias);
              b0 = o < args.O ? __half2float(bp[o]) : 0.f;
              b1 = o + 1 < args.O ? __half2float(bp[o + 1]) : 0.f;
            }
            h[i] = h2_bits(__floats2half2_rn(__uint_as_float(r[2 * i]) + b0,
                                             __uint_as_float(r[2 * i + 1]) + b1));
          }
          ptx::tmem_st_32x32b_x8(park + col / 2, h);
        };
        ptx::tmem_ld_32x32b_x16(taddr, ra);
        for (int col = 0; col < ncols; col += 32) {  // warp-uniform bounds
          ptx::tmem_wait_ld_regs(ra);
          if (col + 16 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 16, rb);
          drain(ra, col);
          if (col + 16 < ncols) {
            ptx::tmem_wait_ld_regs(rb);
            if (col + 32 < ncols) ptx::tmem_ld_32x32b_x16(taddr + col + 32, ra);
            drain(rb, col + 16);
          }
        }
        release();
        ptx::tmem_wait_st();
        // 2) stores of y from the park columns, while the MMAs of the next tile run
        auto store = [&](const uint32_t (&w)[16], int col) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int o = o_chunk + col + 2 * i;  // channels o, o + 1 in word i
            if (paired) {
              // lanes (2j, 2j+1): the even lane stores channel o, the odd one o + 1, both for
              // pixels (pe, pe + 1)
              const uint32_t recv = __shfl_xor_sync(0xffffffffu, w[i], 1);
              const uint32_t pr = odd ? __byte_perm(recv, w[i], 0x7632)
                                      : __byte_perm(w[i], recv, 0x5410);
              if (o + odd < args.O && pe < args.P)
                *reinterpret_cast<uint32_t*>(yimg + static_cast<size_t>(o + odd) * args.P + pe) = pr;
            } else if (p < args.P) {
              if (o < args.O)
                *reinterpret_cast<unsigned short*>(yimg + static_cast<size_t>(o) * args.P + p) =
                    static_cast<unsigned short>(w[i] & 0xFFFFu);
              if (o + 1 < args.O)
                *reinterpret_cast<unsigned short*>(yimg + static_cast<size_t>(o + 1) * args.P + p) =
                    static_cast<unsigned short>(w[i] >> 16);
            }
          }
        };
        ptx::tmem_ld_32x32b_x16(park, ra);
        for (int col = 0; col < ncols; col += 64) {  // 32 channels per load
          ptx::tmem_wait_ld_regs(ra);
          if (col + 32 < ncols) ptx::tmem_ld_32x32b_x16(park + col / 2 + 16, rb);
          store(ra, col);
          if (col + 32 < ncols) {
            ptx::tmem_wait_ld_regs(rb);
            if (col + 64 < ncols) ptx::tmem_ld_32x32b_x16(park + col / 2 + 32, ra);
            store(rb, col + 32);
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
        release();
      }
    }
  } else {
    // ------------------------------------------------------------ samplers
    // Thread = A row (pixel) mrow = 32 * (warp % 4) + lane of the CTA's 128. The 3 warps of a lane
    // quadrant split the taps: warp j = (warp - kSampWarp0) / 4 takes the K-blocks of taps
    // t = j (mod 3) and writes whole 128-byte rows (all 8 chunks: 32 TMEM columns) of them, so it
    // needs the geometry of its own taps only. Per K-block a thread reads the 4 corners of each
    // chunk (32 x 16 bytes), mixes them and stores its row with one tcgen05.st; the store of a
    // K-block is published after the next K-block's loads and mix (one store in flight per warp).
    constexpr int EPC = TR::kChunkElems, KC = TR::kBlockElems, EB = TR::kElemBytes;
    // 3x3 fast path (cached tap geometry, rotated conflict-free corner loads): fp16 with
    // packed-half mix or, PRECISE, with fp32 corner weights and the fp32 mix; int8.
    constexpr bool kFast = KT > 0;
    constexpr int kMyTaps = kFast ? (KT + kTaTapGroups - 1) / kTaTapGroups : 1;
    constexpr uint32_t kNoWin = 0xFFFFu;
    const int sw = warp - kSampWarp0;
    const int q = warp & 3;
    const int j = sw >> 2;  // tap group
    const int mrow = q * 32 + lane;
    constexpr int SAC = TaLayout<PREC>::kAStages;  // power of two
    const uint32_t a_tm = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + TaLayout<PREC>::kACol0;
    const bool issuer = args.use_win && sw == 0 && lane == 0;
    const uint32_t rot16 = static_cast<uint32_t>(lane & 7) << 4;  // fast path: chunk rotation
    const GT* offp = reinterpret_cast<const GT*>(args.offset);
    const GT* maskp = reinterpret_cast<const GT*>(args.mask);
    const uint32_t w_base = ptx::smem_addr(w_smem);
    const int cb_per_tile = args.dg * args.CBg;
    const int T = KT > 0 ? KT : args.T;
    const int K = KT == 9 ? 3 : args.K;
    int kb_seq = 0;    // K-blocks of this CTA before the current channel block
    int cbi = 0;       // channel-block sequence number (window buffer cbi & 1)
    bool ok = true;
    bool pending = false;  // a TMEM store of stage pend_s not yet published
    int pend_s = 0;

    // Loads window qq (the CTA's channel-block sequence number) into buffer qq & 1, which no
    // warp reads any more. One thread.
    auto issue_window = [&](int qq) {
      const int k = qq / cb_per_tile, r = qq - k * cb_per_tile;
      const int tl = tile0 + k * tstep;
      if (tl >= args.num_tiles) return;
      const int g = r / args.CBg, cbg = r - g * args.CBg;
      int im, pt, cc;
      decode_tile(args, tl, im, pt, cc);
      const int row0 = (pix_base(pt) / args.Wo) * args.stride - args.win_top;
      const int b = qq & 1;
      ptx::mbar_arrive_expect_tx(win_full + 8 * b, args.win_bytes);
      ptx::tma_load_4d(w_base + b * args.win_stride, &tmap_x, (g * args.Cg + cbg * KC) * EB, 0,
                       row0, im, win_full + 8 * b);
      atomicMax(win_issued, static_cast<uint32_t>(qq + 1));
    };
    if (issuer) {
      issue_window(0);
      issue_window(1);
    }

    auto prefetch_geometry = [&](int tl) {
      if (tl >= args.num_tiles) return;
      int im, ptn, ccn;
      decode_tile(args, tl, im, ptn, ccn);
      const int p0 = pix_base(ptn);
      const int cnt = args.P - p0 < kTileM ? args.P - p0 : kTileM;
      if (cnt <= 0) return;
      const int bytes = cnt * static_cast<int>(sizeof(GT));
      const int lines = (bytes + 127) / 128 + 1;
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

    // Publishes the pending TMEM store (4 warps, one per quadrant, arrive once per stage).
    auto flush = [&]() {
      if (pending) {
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(a_full + 8 * pend_s);
        pending = false;
      }
    };
    // Publishes the previous K-block and waits until the stage of K-block kb (CTA sequence
    // number) is free; returns its first TMEM column address for this warp's lanes.
    auto acquire = [&](int kb, uint32_t& ta) -> bool {
      flush();
      const int s = kb & (SAC - 1);
      const uint32_t ph = static_cast<uint32_t>(kb / SAC) & 1u;
      const bool got = wait_bar<kSuspend>(a_empty + 8 * s, ph ^ 1u, wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
      if (!__all_sync(0xffffffffu, got)) return false;
      ptx::tc_fence_after();
      ta = a_tm + static_cast<uint32_t>(s) * kTaStageCols;
      pend_s = s;
      return true;
    };

    for (int tile = tile0; tile < args.num_tiles && ok; tile += tstep) {
      int img, pt, cc;
      decode_tile(args, tile, img, pt, cc);
      const int my_pix = pix_base(pt) + mrow;
      const bool my_val = my_pix < args.P;
      const int pcl = my_val ? my_pix : 0;
      const int oh = pcl / args.Wo, ow = pcl - (pcl / args.Wo) * args.Wo;
      const int my_bh = oh * args.stride - args.pad;
      const int my_bw = ow * args.stride - args.pad;
      const int row0 = (pix_base(pt) / args.Wo) * args.stride - args.win_top;
      const uint8_t* ximg = args.x_nhwc + static_cast<size_t>(img) * args.H * args.W * args.C * EB;
      if (sw == 0) prefetch_geometry(tile + tstep);

      auto geom = [&](int g, int t, int comp) -> float {
        const size_t ig = static_cast<size_t>(img) * args.dg + g;
        return comp < 2 ? load_geom_value(offp + (ig * 2 * args.T + 2 * t + comp) * args.P + my_pix)
                        : load_geom_value(maskp + (ig * args.T + t) * args.P + my_pix);
      };

      for (int g = 0; g < args.dg && ok; ++g) {
        // the MMA may be waiting for this warp's last stage while the geometry loads run
        flush();
        // fast path (3x3): the 4 corners of each of this warp's taps as
        // (16-bit weight | window byte offset of the corner pixel << 16)
        uint32_t cw[kMyTaps][4];
        float cwf[PRECISE ? kMyTaps : 1][4];  // PRECISE: the fp32 corner weights
        bool fast_g = false;
        if (kFast) {
          float gv[3 * kMyTaps];
#pragma unroll
          for (int u = 0; u < kMyTaps; ++u) {
            const int t = j + kTaTapGroups * u;
#pragma unroll
            for (int i = 0; i < 3; ++i) gv[3 * u + i] = (my_val && t < T) ? geom(g, t, i) : 0.f;
            if (PREC == PREC_I8) gv[3 * u + 2] = i8_mask(gv[3 * u + 2]);
          }
          bool inwin = true;
#pragma unroll
          for (int u = 0; u < kMyTaps; ++u) {
            const int t = j + kTaTapGroups * u;
            const int ki = t / K, kj = t - ki * K;
            float wt[4];
            int loc[4];
            ta_tap_geom(args, my_val, my_bh + ki * args.dil, my_bw + kj * args.dil, gv[3 * u],
                        gv[3 * u + 1], gv[3 * u + 2], row0, wt, loc);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              inwin = inwin && (t >= T || loc[c] >= 0);
              // fp16: the weight's fp16 bits; int8: its 16-bit fixed-point value; PRECISE: the
              // fp32 weight is kept beside the word
              const uint32_t hb =
                  PRECISE ? 0u
                  : PREC == PREC_F16 ? static_cast<uint32_t>(__half_as_ushort(__float2half_rn(wt[c])))
                                     : i8_weight(wt[c]);
              if constexpr (PRECISE) cwf[u][c] = wt[c];
              cw[u][c] = hb | ((loc[c] >= 0 ? static_cast<uint32_t>(loc[c]) : kNoWin) << 16);
            }
          }
          fast_g = __all_sync(0xffffffffu, inwin);
        }
        const int gbase = g * args.Cg;
        for (int cbg = 0; cbg < args.CBg && ok; ++cbg) {
          const int b = cbi & 1;
          if (args.use_win) {
            const bool got = wait_bar<kSuspend>(win_full + 8 * b, static_cast<uint32_t>(cbi >> 1) & 1u,
                                                wc, DCNV2_DEVERR_TIMEOUT_SAMPLER);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
          }
          const uint32_t win = w_base + b * args.win_stride;
          const bool all_valid = (cbg + 1) * KC <= args.Cg;  // block-uniform
          if (kFast && fast_g && all_valid) {
#pragma unroll
            for (int u = 0; u < kMyTaps; ++u) {
              const int t = j + kTaTapGroups * u;
              if (t >= T) break;
              __half2 wh[4];
              uint32_t pix[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const uint32_t v = cw[u][c];
                pix[c] = win + (v >> 16);  // the corner pixel's 128 bytes
                wh[c] = __half2half2(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
              }
              // int8: weight pairs (w0 | w1 << 16), (w2 | w3 << 16) for dp2a
              const uint32_t w01 = __byte_perm(cw[u][0], cw[u][1], 0x5410);
              const uint32_t w23 = __byte_perm(cw[u][2], cw[u][3], 0x5410);
              // step h: chunk h ^ rot of every corner (conflict-free phases), mixed into out[4h..]
              uint32_t out[32];
              // int8: the loads of chunk h + 1 are issued before chunk h is mixed (its integer
              // mix is long enough to cover their latency)
              uint4 xn[4];
              if constexpr (PREC == PREC_I8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) xn[c] = ptx::ld_shared_v4(pix[c] + rot16);
              }
#pragma unroll
              for (int h = 0; h < 8; ++h) {
                const uint32_t co = (static_cast<uint32_t>(h) << 4) ^ rot16;
                uint4 xv[4];
                if constexpr (PREC == PREC_I8) {
#pragma unroll
                  for (int c = 0; c < 4; ++c) xv[c] = xn[c];
                  if (h + 1 < 8) {
                    const uint32_t cn = (static_cast<uint32_t>(h + 1) << 4) ^ rot16;
#pragma unroll
                    for (int c = 0; c < 4; ++c) xn[c] = ptx::ld_shared_v4(pix[c] + cn);
                  }
                } else {
#pragma unroll
                  for (int c = 0; c < 4; ++c) xv[c] = ptx::ld_shared_v4(pix[c] + co);
                }
                // the previous K-block's TMEM store has had time to land: publish it now rather
                // than after this whole K-block
                if (h == 0) flush();
                if (PREC == PREC_F16 && PRECISE) {
                  out[4 * h + 0] = f16_mix_precise(cwf[u], xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[4 * h + 1] = f16_mix_precise(cwf[u], xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[4 * h + 2] = f16_mix_precise(cwf[u], xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[4 * h + 3] = f16_mix_precise(cwf[u], xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                } else if (PREC == PREC_F16) {
                  out[4 * h + 0] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[4 * h + 1] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[4 * h + 2] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[4 * h + 3] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                } else {
                  out[4 * h + 0] = i8_mix_fx(w01, w23, xv[0].x, xv[1].x, xv[2].x, xv[3].x);
                  out[4 * h + 1] = i8_mix_fx(w01, w23, xv[0].y, xv[1].y, xv[2].y, xv[3].y);
                  out[4 * h + 2] = i8_mix_fx(w01, w23, xv[0].z, xv[1].z, xv[2].z, xv[3].z);
                  out[4 * h + 3] = i8_mix_fx(w01, w23, xv[0].w, xv[1].w, xv[2].w, xv[3].w);
                }
                // chunk h is mixed before the loads of chunk h + 1 are issued
                asm volatile("" : "+r"(out[4 * h + 0]), "+r"(out[4 * h + 1]),
                             "+r"(out[4 * h + 2]), "+r"(out[4 * h + 3]));
              }
              unrotate_chunks(out, lane & 7);
              uint32_t ta = 0;
              if (!acquire(kb_seq + t, ta)) { ok = false; break; }
              ptx::tmem_st_32x32b_x32(ta, out);
              if (!ok) break;
              pending = true;
            }
          } else {
            // General path: geometry of the tap per K-block, corners from the window or from
            // global memory, partial channel chunks zero.
            for (int t = j; t < T && ok; t += kTaTapGroups) {
              const int ki = t / K, kj = t - ki * K;
              float dh = 0.f, dw = 0.f, m = 0.f;
              if (my_val) {
                dh = geom(g, t, 0);
                dw = geom(g, t, 1);
                m = geom(g, t, 2);
                if (PREC == PREC_I8) m = i8_mask(m);
              }
              float wt[4];
              int loc[4];
              ta_tap_geom(args, my_val, my_bh + ki * args.dil, my_bw + kj * args.dil, dh, dw, m,
                          row0, wt, loc);
              __half2 wh[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) wh[c] = __half2half2(__float2half_rn(wt[c]));
              uint32_t ta = 0;
#pragma unroll
              for (int half = 0; half < 2; ++half) {
              uint32_t out[16];
#pragma unroll
              for (int hh = 0; hh < 4; ++hh) {
                const int h = 4 * half + hh;
                const int cig = cbg * KC + h * EPC;  // channel within the group
                const bool cvalid = cig < args.Cg;
                uint4 xv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int e = loc[c];
                  if (!cvalid) {
                    xv[c] = make_uint4(0, 0, 0, 0);
                  } else if (e >= 0) {
                    xv[c] = ptx::ld_shared_v4(win + (static_cast<uint32_t>(e) ^ (h << 4)));
                  } else {
                    xv[c] = ptx::ld_nc_v4(ximg + (static_cast<size_t>(-e - 1) * args.C + gbase + cig) * EB);
                  }
                }
                const uint4& x0 = xv[0];
                const uint4& x1 = xv[1];
                const uint4& x2 = xv[2];
                const uint4& x3 = xv[3];
                if (PREC == PREC_F16 && !PRECISE) {
                  out[4 * hh + 0] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], x0.x, x1.x, x2.x, x3.x);
                  out[4 * hh + 1] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], x0.y, x1.y, x2.y, x3.y);
                  out[4 * hh + 2] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], x0.z, x1.z, x2.z, x3.z);
                  out[4 * hh + 3] = f16_mix_h2(wh[0], wh[1], wh[2], wh[3], x0.w, x1.w, x2.w, x3.w);
                } else if (PREC == PREC_F16) {
                  out[4 * hh + 0] = f16_mix_precise(wt, x0.x, x1.x, x2.x, x3.x);
                  out[4 * hh + 1] = f16_mix_precise(wt, x0.y, x1.y, x2.y, x3.y);
                  out[4 * hh + 2] = f16_mix_precise(wt, x0.z, x1.z, x2.z, x3.z);
                  out[4 * hh + 3] = f16_mix_precise(wt, x0.w, x1.w, x2.w, x3.w);
                } else {
                  out[4 * hh + 0] = i8_mix_word(wt, x0.x, x1.x, x2.x, x3.x);
                  out[4 * hh + 1] = i8_mix_word(wt, x0.y, x1.y, x2.y, x3.y);
                  out[4 * hh + 2] = i8_mix_word(wt, x0.z, x1.z, x2.z, x3.z);
                  out[4 * hh + 3] = i8_mix_word(wt, x0.w, x1.w, x2.w, x3.w);
                }
              }
              if (half == 0 && !acquire(kb_seq + t, ta)) { ok = false; break; }
              ptx::tmem_st_32x32b_x16(ta + 16 * half, out);
              }
              if (!ok) break;
              pending = true;
            }
          }
          if (!ok) break;
          if (args.use_win) {
            // every corner load of this channel block has returned (its values are mixed); the
            // last warp to finish with the buffer loads the window two channel blocks ahead
            // into it, so no warp waits for the others here
            __syncwarp();
            if (lane == 0) {
              __threadfence_block();
              const uint32_t uses = static_cast<uint32_t>(cbi >> 1) + 1u;
              if (atomicAdd(win_done + b, 1u) == uses * kTaSampWarps - 1u) {
                __threadfence_block();
                ptx::fence_proxy_async_smem();
                issue_window(cbi + 2);
              }
            }
          }
          ++cbi;
          kb_seq += T;
        }
      }
    }
    if (ok) flush();
    else if (pending) ptx::tmem_wait_st();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (args.use_win && warp == kSampWarp0 && lane == 0) {
    // window loads still in flight (after an early exit) land before shared memory is released
    const int issued = static_cast<int>(*reinterpret_cast<volatile uint32_t*>(win_issued));
    for (int qq = issued - 2 < 0 ? 0 : issued - 2; qq < issued; ++qq)
      wait_bar(win_full + 8 * (qq & 1), static_cast<uint32_t>(qq >> 1) & 1u, wc,
               DCNV2_DEVERR_TIMEOUT_DRAIN);
  }
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTaTmemCols);
  }
}

}  // namespace dcnv2
