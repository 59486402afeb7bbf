// dcnv2_head_kernel.cuh — the offset / mask head of a DCNv2 block on tensor cores.
//
// A DCNv2 block computes its sampling offsets and mask from its own input with a plain
// convolution: om = Conv2d(C -> 3*dg*K*K, K x K, stride 1, padding (K-1)/2)(x), offset =
// om[:, :2*dg*K*K], mask = sigmoid(om[:, 2*dg*K*K:]) (the reference's DCNBlock,
// python/detector.py:44,50-52; python/01_oracle_and_export.py:42,46-48). This kernel computes
// that head from the channels-last copy of x the DCNv2 forward writes anyway, and stores offset
// and mask in the layout the deformable kernels read, so the head adds no NCHW pass over x and
// no separate split / sigmoid pass.
//
// Implicit GEMM per tile of 128 output pixels (TR rows x TW columns): D[128, n_head] =
// A[128, C*K*K] * B[n_head, C*K*K]^T with K ordered (channel block of 64, tap) as the packed
// weights of pack_weights_kernel. The A tile of K-block (cb, tap) is one 4-D TMA box of the
// channels-last x, shifted by the tap and swizzled by the tensor map (128-byte swizzle): it lands
// in shared memory exactly as the MMA descriptor reads it, and the box's out-of-image part reads
// zeros, which is the convolution's zero padding. No sampler threads are involved.
//
// Window mode (TW a multiple of 8 and two stages fit): a stage is one channel block — K TMA
// boxes of (TR + K - 1) rows x TW columns, box kj shifted by the tap column kj, plus one bulk copy
// of the block's K*K weight tiles. The A tile of tap (ki, kj) is rows [ki*TW, ki*TW + 128) of box
// kj: it starts on a 1024-byte swizzle atom (TW*128 is a multiple of 1024), so the same
// descriptor reads it. Per channel block that is K*(TR+K-1)*TW line requests instead of
// K*K*TR*TW (3x3, 8 x 16 tiles: 480 instead of 1152).
//
// Roles (192 threads): warp 0 producer (TMA box of A + bulk copy of B per K-block into a ring of
// stages), warp 1 MMA issuer (tcgen05.mma kind::f16, fp32 accumulators in TMEM, two of them so
// that the epilogue of a tile overlaps the next tile), warps 2-5 epilogue (tcgen05.ld, + bias,
// offsets stored as fp16, sigmoid of the mask channels stored as fp16). Every wait is bounded.
#pragma once
#include "dcnv2_kernels.cuh"

namespace dcnv2 {

constexpr int kHeadThreads = (kEpiWarp0 + kNumEpiWarps) * 32;  // 192
constexpr int kHeadMaxStages = 8;
constexpr uint32_t kHeadABytes = kTileM * kRowBytes;             // 16 KB: 128 pixels x 64 fp16

struct HeadArgs {
  const uint8_t* wpack;   // [numKB][n_mma rows][128 B], pre-swizzled (pack_weights_kernel)
  const __half* bias;     // [n_head] or null
  __half* offset;         // [N][n_off][H][W]
  __half* mask;           // [N][n_head - n_off][H][W]
  int* err;               // device error word
  int N, C, H, W;
  int K, pad;             // head kernel size and padding (stride 1, dilation 1: Ho = H)
  int n_head, n_off, n_mma;
  int numKB, T;           // numKB = channel blocks * T, T = K*K taps
  int TW, TR;             // tile: TR rows x TW columns, TR * TW = 128
  int tiles_x, tiles_y, num_tiles;
  int stages;
  uint32_t b_stage_bytes, tmem_cols;  // b_stage_bytes: one K-block's weight tile
  int win_mode;                        // 1: a stage holds a channel block's K windows + T tiles
  uint32_t win_bytes;                  // window mode: one box, (TR + K - 1) * TW * 128 bytes
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void head_tile(const HeadArgs& a, int tile, int& img, int& oy0,
                                          int& ox0) {
  const int per_img = a.tiles_x * a.tiles_y;
  img = tile / per_img;
  const int r = tile - img * per_img;
  oy0 = (r / a.tiles_x) * a.TR;
  ox0 = (r - (r / a.tiles_x) * a.tiles_x) * a.TW;
}

__global__ void __launch_bounds__(kHeadThreads, 1)
    dcnv2_offset_head_kernel(const HeadArgs args, const __grid_constant__ CUtensorMap tmap_x) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.stages;
  // [S A stages (1 KB aligned) | S B stages | barriers]; per stage A is one 16 KB box (tap mode)
  // or K windows (window mode), B one weight tile (tap mode) or the T tiles of a channel block
  const uint32_t a_bytes = args.win_mode ? static_cast<uint32_t>(args.K) * args.win_bytes
                                         : kHeadABytes;
  const uint32_t b_bytes = args.win_mode ? static_cast<uint32_t>(args.T) * args.b_stage_bytes
                                         : args.b_stage_bytes;
  const int n_steps = args.win_mode ? args.numKB / args.T : args.numKB;  // stages per tile
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + static_cast<size_t>(S) * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_smem + static_cast<size_t>(S) * b_bytes);
  const uint32_t full = ptx::smem_addr(bars);     // [S] A and B of a stage landed
  const uint32_t empty = full + 8 * S;            // [S] MMAs of a stage done
  const uint32_t tfull = empty + 8 * S;           // [2] accumulator ready
  const uint32_t tempty = tfull + 16;             // [2] accumulator read by the epilogue
  const uint32_t drain = tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const WaitCtx wc{args.timeout_ns, args.err, abort_flag};
  ptx::griddep_launch_dependents();  // the layer's main kernel may come up on free SMs

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(full + 8 * s, 1);
      ptx::mbar_init(empty + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(tfull + 8 * i, 1);
      ptx::mbar_init(tempty + 8 * i, kNumEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), args.tmem_cols);
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
    // ------------------------------------------------------------ producer (A box + B tile)
    if (lane == 0) {
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t a_base = ptx::smem_addr(a_smem), b_base = ptx::smem_addr(b_smem);
      for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x) {
        int img, oy0, ox0;
        head_tile(args, tile, img, oy0, ox0);
        for (int step = 0; step < n_steps; ++step, ++it) {
          if (!wait_bar<kSuspend>(empty + 8 * s, ph ^ 1u, wc, DCNV2_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(full + 8 * s, a_bytes + b_bytes);
          if (args.win_mode) {
            // channel block `step`: K windows, box kj shifted by the tap column kj
            for (int kj = 0; kj < args.K; ++kj)
              ptx::tma_load_4d(a_base + s * a_bytes + kj * args.win_bytes, &tmap_x,
                               step * kRowBytes, ox0 + kj - args.pad, oy0 - args.pad, img,
                               full + 8 * s);
            ptx::bulk_copy_g2s(b_base + s * b_bytes,
                               args.wpack + static_cast<size_t>(step) * b_bytes, b_bytes,
                               full + 8 * s);
          } else {
            const int kb = step, t = kb % args.T, cb = kb / args.T;
            const int ki = t / args.K, kj = t - ki * args.K;
            // channel block cb (128 bytes, 16-byte aligned), columns and rows shifted by the tap
            ptx::tma_load_4d(a_base + s * a_bytes, &tmap_x, cb * kRowBytes, ox0 + kj - args.pad,
                             oy0 + ki - args.pad, img, full + 8 * s);
            ptx::bulk_copy_g2s(b_base + s * b_bytes,
                               args.wpack + static_cast<size_t>(kb) * b_bytes, b_bytes,
                               full + 8 * s);
          }
          if (++s == S) { s = 0; ph ^= 1u; }
        }
      }
      // copies still in flight (at most the last one per stage) land before the CTA exits
      const int outstanding = it < S ? it : S;
      for (int j = 0; j < outstanding; ++j) {
        const int idx = it - 1 - j;
        wait_bar(full + 8 * (idx % S), (idx / S) & 1, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::make_idesc(1, 0, static_cast<uint32_t>(args.n_mma), kTileM);
      const uint64_t desc0 = ptx::sw128_kmajor_desc(0);
      const uint32_t a_base = ptx::smem_addr(a_smem), b_base = ptx::smem_addr(b_smem);
      int s = 0, acc = 0;
      uint32_t ph = 0, use = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x) {
        if (!wait_bar<kSuspend>(tempty + 8 * acc, use ^ 1u, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * args.n_mma);
        for (int step = 0; step < n_steps; ++step) {
          if (!wait_bar(full + 8 * s, ph, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const int taps = args.win_mode ? args.T : 1;
          for (int t = 0; t < taps; ++t) {
            // window mode: tap (ki, kj) reads rows [ki*TW, ki*TW + 128) of window kj
            const int ki = t / args.K, kj = t - ki * args.K;
            const uint32_t a_addr = a_base + s * a_bytes +
                                    (args.win_mode ? kj * args.win_bytes +
                                                         static_cast<uint32_t>(ki * args.TW) * kRowBytes
                                                   : 0u);
            const uint32_t b_addr = b_base + s * b_bytes + t * args.b_stage_bytes;
            const uint64_t ad = desc0 | ((a_addr >> 4) & 0x3FFFu);
            const uint64_t bd = desc0 | ((b_addr >> 4) & 0x3FFFu);
#pragma unroll
            for (int k = 0; k < 4; ++k)  // K-step k: 32 bytes further along the rows
              ptx::mma_f16(d, ad + 2 * k, bd + 2 * k, idesc,
                           (step > 0 || t > 0 || k > 0) ? 1u : 0u);
          }
          ptx::tc_commit(empty + 8 * s);
          if (++s == S) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        ptx::tc_commit(tfull + 8 * acc);
        if (++acc == 2) { acc = 0; use ^= 1u; }
      }
      ptx::tc_commit(drain);
      wait_bar(drain, 0, wc, DCNV2_DEVERR_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Thread = pixel m = 32 * (warp % 4) + lane of the tile (TMEM lane m), column tw = m % TW,
    // row tr = m / TW. Channels c < n_off are offsets, the rest mask logits.
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const int tr = m / args.TW, tw = m - (m / args.TW) * args.TW;
    const size_t plane = static_cast<size_t>(args.H) * args.W;
    const int n_msk = args.n_head - args.n_off;
    int tl = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++tl) {
      const int acc = tl & 1;
      const uint32_t ph = static_cast<uint32_t>(tl >> 1) & 1u;
      const bool got = wait_bar<kSuspend>(tfull + 8 * acc, ph, wc, DCNV2_DEVERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      ptx::tc_fence_after();
      int img, oy0, ox0;
      head_tile(args, tile, img, oy0, ox0);
      const int oy = oy0 + tr, ox = ox0 + tw;
      const bool valid = oy < args.H && ox < args.W;
      const size_t pix = static_cast<size_t>(oy) * args.W + ox;
      __half* off_img = args.offset + static_cast<size_t>(img) * args.n_off * plane;
      __half* msk_img = args.mask + static_cast<size_t>(img) * n_msk * plane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * args.n_mma);
      for (int col = 0; col < args.n_head; col += 16) {  // warp-uniform bound
        uint32_t r[16];
        ptx::tmem_ld_32x32b_x16(taddr + col, r);
        ptx::tmem_wait_ld_regs(r);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = col + i;
            if (c < args.n_head) {
              const float v = __uint_as_float(r[i]) + (args.bias ? __half2float(args.bias[c]) : 0.f);
              if (c < args.n_off) off_img[static_cast<size_t>(c) * plane + pix] = __float2half_rn(v);
              else msk_img[static_cast<size_t>(c - args.n_off) * plane + pix] =
                       __float2half_rn(1.f / (1.f + __expf(-v)));
            }
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(tempty + 8 * acc);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, args.tmem_cols);
  }
}

}  // namespace dcnv2
