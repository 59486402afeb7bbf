// dcnv2_api.cu — host side of libdcnv2.so: validation, the launch plan (tile shape, pipeline
// depth, TMEM columns, workspace layout) and the stateless C ABI declared in include/dcnv2.h.
//
// Replaces the dispatch in DCNv2Plugin::enqueue (src/dcn_plugin.cpp:122-176) and the workspace
// rule of getWorkspaceSize (:110-118). Differences from the reference, all deliberate:
//   * every image of the batch is computed (the reference reads only image 0, :125-130);
//   * deformable_groups is honoured (the reference stores it but never uses it, :197);
//   * the workspace holds a channels-last copy of x and the packed weights instead of the
//     fp32 column matrix, and it scales with N;
//   * failures are reported as dcnv2_status values (the reference returns 0 unconditionally).
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/dcnv2.h"
#include "../../include/dcnv2_diag.h"
#include <cudaTypedefs.h>
#include "dcnv2_head_kernel.cuh"
#include "dcnv2_kernels.cuh"
#include "dcnv2_ta_kernel.cuh"

namespace dcnv2 {

namespace {

constexpr size_t kSmemLimit = 227 * 1024;     // opt-in dynamic shared memory per block
constexpr size_t kErrBytes = 256;
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // 2 s per on-chip wait

struct DevInfo {
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  bool ok = false;
  std::atomic<uint32_t> attr_set{0};
  std::atomic<int> pair_clusters[3] = {{0}, {0}, {0}};  // co-resident CTA pairs, per precision
};
constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

DevInfo* device_info(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_dev_once[dev], [dev]() {
    DevInfo& d = g_dev[dev];
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      cudaGetLastError();
      d.ok = false;
      return;
    }
    d.ok = true;
  });
  return &g_dev[dev];
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Kernel-selection overrides for measurements and tests. They are read from the environment
// once per process (DCNV2_KERNEL=ta|smem, DCNV2_PAIR=1|0) and can be changed afterwards only
// through dcnv2_diag_set_kernel_override; the dispatch itself never calls getenv.
enum { KOV_AUTO = 0, KOV_TA = 1, KOV_SMEM = 2 };
enum { POV_AUTO = 0, POV_PAIRS = 1, POV_SINGLE = 2 };
std::atomic<int> g_kernel_override{KOV_AUTO};
std::atomic<int> g_pair_override{POV_AUTO};
std::once_flag g_env_once;
void read_env_overrides() {
  std::call_once(g_env_once, []() {
    const char* ke = std::getenv("DCNV2_KERNEL");
    if (ke && std::strcmp(ke, "smem") == 0) g_kernel_override.store(KOV_SMEM);
    else if (ke && std::strcmp(ke, "ta") == 0) g_kernel_override.store(KOV_TA);
    const char* pe = std::getenv("DCNV2_PAIR");
    if (pe && pe[0] == '1' && pe[1] == 0) g_pair_override.store(POV_PAIRS);
    else if (pe && pe[0] == '0' && pe[1] == 0) g_pair_override.store(POV_SINGLE);
  });
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    cudaGetLastError();
  });
  return fn;
}

// Optional CUDA events recorded between the launches of one forward (diagnostics only).
struct Marks {
  void* const* ev = nullptr;
  int n = 0;
  int i = 0;
  void mark(cudaStream_t st) {
    if (ev && i < n) cudaEventRecord(static_cast<cudaEvent_t>(ev[i++]), st);
  }
};
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

enum Kind { KIND_SIMT = 0, KIND_TCGEN05 = 1, KIND_F32_EXACT = 2 };

struct Plan {
  int prec = 0;
  int kind = KIND_SIMT;
  bool fused = false;  // kind == KIND_TCGEN05
  int N, C, H, W, O, K, T, stride, pad, dil, dg, Ho, Wo, P, Cg;
  int elem_bytes;
  // fused-kernel configuration
  int CBg = 0, numKB = 0, cchunks = 0, nrows = 0, nsub = 0, n_mma = 0, acc_bufs = 0;
  int stages = 0, tiles_per_img = 0, num_tiles = 0;
  bool pair = false;  // CTA pairs (cta_group::2), tiles of 256 pixels
  uint32_t tmem_cols = 0, a_stage_bytes = 0, b_stage_bytes = 0;  // per CTA
  size_t b_kb_bytes = 0;  // packed weights of one K-block (both halves of a pair)
  size_t smem_bytes = 0;
  uint32_t epi_off = 0;   // TMA-store staging of the epilogue (A-in-shared-memory kernel), 0: none
  // fp32-exact kernel configuration
  int x_ptiles = 0, x_ctiles = 0;
  // workspace layout (offsets from the 256-byte aligned base)
  size_t off_x = 0, off_w = 0, ws_bytes = 0;
  // shared-memory window of x for the fused kernel (two buffers of win_bytes)
  bool use_win = false;
  int win_rows = 0, win_top = 0;
  uint32_t win_bytes = 0;
  bool tf32_single = false, precise = false, i8_rint = false;
  // A operand in TMEM (dcnv2_fused_ta_kernel): A ring in TMEM, B ring in shared memory
  bool ta = false;
  int a_stages = 0, b_stages = 0;
  uint32_t win_stride = 0;
  // int8 groups of 64 channels (half of a 128-byte K-block): two taps per K-block
  bool tap_pairs = false;
};

int prec_of(int dtype) {
  switch (dtype) {
    case DCNV2_FLOAT: return PREC_F32;
    case DCNV2_HALF: return PREC_F16;
    case DCNV2_INT8: return PREC_I8;
    default: return -1;
  }
}

int elem_bytes_of(int prec) { return prec == PREC_F32 ? 4 : prec == PREC_F16 ? 2 : 1; }
int chunk_elems_of(int prec) { return prec == PREC_F32 ? 4 : prec == PREC_F16 ? 8 : 16; }
int block_elems_of(int prec) { return prec == PREC_F32 ? 32 : prec == PREC_F16 ? 64 : 128; }

// Largest number of output rows of a tile of `tile_px` consecutive output pixels (whole image
// scan for up to 4096 tiles; beyond that with Wo > 4096 no exact bound is taken).
int max_tile_rows(const Plan& p, int tile_px) {
  const int64_t P = int64_t(p.Ho) * p.Wo;
  const int64_t tiles = (P + tile_px - 1) / tile_px;
  int rows_max = 0;
  const int64_t loop = tiles < 4096 ? tiles : 4096;
  for (int64_t pt = 0; pt < loop; ++pt) {
    const int64_t a0 = pt * tile_px, a1 = (a0 + tile_px < P ? a0 + tile_px : P) - 1;
    const int rows = static_cast<int>(a1 / p.Wo - a0 / p.Wo + 1);
    if (rows > rows_max) rows_max = rows;
  }
  if (tiles > 4096 && p.Wo > 4096) rows_max = 1 << 20;
  return rows_max;
}

// Configuration of dcnv2_fused_ta_kernel: one accumulator of n_mma <= 256 columns and up to 8
// A stages of 32 columns in 512 TMEM columns; shared memory holds two x windows (1 KB aligned)
// and the B ring. The window covers, for every pixel of a CTA's 128, the taps
// whose offsets lie in (-1 - M, 1 + M) for the largest margin M <= 2 that still leaves three B
// stages (else two); corners outside it are read from global memory.
void plan_ta(Plan* pl) {
  Plan& p = *pl;
  p.ta = true;
  p.cchunks = static_cast<int>(cdiv(p.O, 256));
  p.nsub = 1;
  p.n_mma = static_cast<int>(cdiv(cdiv(p.O, p.cchunks), 16) * 16);
  p.nrows = p.n_mma;
  p.acc_bufs = 1;
  p.tmem_cols = kTaTmemCols;
  p.a_stages = p.prec == PREC_F16 ? TaLayout<PREC_F16>::kAStages : TaLayout<PREC_I8>::kAStages;
  p.a_stage_bytes = 0;
  p.b_kb_bytes = size_t(p.nrows) * kRowBytes;
  p.b_stage_bytes = static_cast<uint32_t>(p.b_kb_bytes);
  p.tiles_per_img = static_cast<int>(cdiv(int64_t(p.Ho) * p.Wo, kTileM));
  p.num_tiles = static_cast<int>(int64_t(p.N) * p.tiles_per_img * p.cchunks);
  const size_t fixed = 1024 + 512 + 1024;  // alignment slack, barriers, staged bias (fp32)
  const size_t per_stage = p.b_stage_bytes;
  auto b_stages_for = [&](size_t win_total) {
    int sb = static_cast<int>((kSmemLimit - fixed - win_total) / per_stage);
    return sb > kTaMaxBStages ? kTaMaxBStages : sb;
  };
  p.use_win = false;
  p.win_rows = 0; p.win_top = 0; p.win_bytes = 0; p.win_stride = 0;
  p.b_stages = b_stages_for(0);
  if (p.W <= 256) {
    const int rows_max = max_tile_rows(p, kTileM);
    const int64_t base = int64_t(rows_max - 1) * p.stride + int64_t(p.K - 1) * p.dil + 3;
    bool done = false;
    for (int want = 3; want >= 2 && !done; --want) {
      for (int M = 2; M >= 0; --M) {
        const int64_t rows = base + 2 * M;
        if (rows > 256) continue;
        const size_t wb = size_t(rows) * p.W * kRowBytes;
        if (wb > 65536) continue;  // window byte offsets travel in 16 bits
        const size_t stride = align_up(wb, 1024);
        if (2 * stride + fixed + size_t(want) * per_stage > kSmemLimit) continue;
        p.use_win = true;
        p.win_rows = static_cast<int>(rows);
        p.win_top = p.pad + 1 + M;
        p.win_bytes = static_cast<uint32_t>(wb);
        p.win_stride = static_cast<uint32_t>(stride);
        p.b_stages = b_stages_for(2 * stride);
        done = true;
        break;
      }
    }
  }
  if (p.b_stages < 2) {
    p.ta = false;  // not reached for nrows <= 256 (32 KB stages); the caller keeps its plan
    return;
  }
  p.stages = p.b_stages;
  p.smem_bytes = fixed + (p.use_win ? 2 * size_t(p.win_stride) : 0) +
                 size_t(p.b_stages) * per_stage;
}

dcnv2_status make_plan(const dcnv2_desc* d, Plan* pl) {
  if (!d || !pl) return DCNV2_ERR_INVALID_ARG;
  read_env_overrides();
  if (d->n < 1 || d->c < 1 || d->h < 1 || d->w < 1 || d->out_c < 1 || d->kernel < 1 ||
      d->stride < 1 || d->padding < 0 || d->dilation < 1 || d->deformable_groups < 1)
    return DCNV2_ERR_INVALID_ARG;
  if (d->c % d->deformable_groups) return DCNV2_ERR_INVALID_ARG;
  if (d->math < DCNV2_MATH_DEFAULT || d->math > DCNV2_MATH_TF32X3) return DCNV2_ERR_INVALID_ARG;
  const int prec = prec_of(d->dtype);
  if (prec < 0) return DCNV2_ERR_UNSUPPORTED;
  if ((d->math == DCNV2_MATH_TF32 || d->math == DCNV2_MATH_TF32X3) && prec != PREC_F32)
    return DCNV2_ERR_INVALID_ARG;
  if (d->math == DCNV2_MATH_PRECISE && prec == PREC_F32) return DCNV2_ERR_INVALID_ARG;
  const int64_t ho = (int64_t(d->h) + 2 * int64_t(d->padding) -
                      int64_t(d->dilation) * (d->kernel - 1) - 1);
  const int64_t wo = (int64_t(d->w) + 2 * int64_t(d->padding) -
                      int64_t(d->dilation) * (d->kernel - 1) - 1);
  if (ho < 0 || wo < 0) return DCNV2_ERR_INVALID_ARG;
  Plan& p = *pl;
  p.prec = prec;
  p.N = d->n; p.C = d->c; p.H = d->h; p.W = d->w; p.O = d->out_c; p.K = d->kernel;
  p.T = d->kernel * d->kernel; p.stride = d->stride; p.pad = d->padding; p.dil = d->dilation;
  p.dg = d->deformable_groups; p.Cg = d->c / d->deformable_groups;
  p.Ho = static_cast<int>(ho / d->stride + 1);
  p.Wo = static_cast<int>(wo / d->stride + 1);
  p.elem_bytes = elem_bytes_of(prec);
  const int64_t P = int64_t(p.Ho) * p.Wo;
  const int64_t plane = int64_t(p.H) * p.W * p.C;
  // 32-bit index limits inside one image (the batch index is 64-bit everywhere).
  if (P >= (int64_t(1) << 31) || plane >= (int64_t(1) << 31) ||
      int64_t(p.O) * P >= (int64_t(1) << 31) || int64_t(p.T) * p.dg * 2 >= (int64_t(1) << 31) ||
      int64_t(p.O) * p.C * p.T >= (int64_t(1) << 31))
    return DCNV2_ERR_INVALID_ARG;
  p.P = static_cast<int>(P);
  p.tf32_single = (d->math == DCNV2_MATH_TF32);
  p.precise = (d->math == DCNV2_MATH_PRECISE) && prec == PREC_F16;

  const bool cg_ok = p.Cg % chunk_elems_of(prec) == 0;
  // fp32 defaults to the fp32-exact CUDA-core fused kernel; the tensor-core kinds of fp32 are
  // opt-in (TF32, TF32X3) because their accumulation error exceeds fp32 rounding.
  const bool f32_exact = prec == PREC_F32 && d->math == DCNV2_MATH_DEFAULT && cg_ok;
  // int8 with DCNV2_MATH_PRECISE: the reference-rounding column rule on the per-output kernel
  p.i8_rint = prec == PREC_I8 && d->math == DCNV2_MATH_PRECISE;
  p.fused = (d->math != DCNV2_MATH_SIMT) && cg_ok && !f32_exact && !p.i8_rint;
  if (f32_exact) {
    p.kind = KIND_F32_EXACT;
    p.CBg = static_cast<int>(cdiv(p.Cg, kXK));
    const int64_t numKB = int64_t(p.dg) * p.T * p.CBg;
    const int64_t ptiles = cdiv(P, kXPx), ctiles = cdiv(p.O, kXCo);
    if (numKB >= (int64_t(1) << 31) || int64_t(p.N) * ptiles * ctiles >= (int64_t(1) << 31)) {
      p.kind = KIND_SIMT;
    } else {
      p.numKB = static_cast<int>(numKB);
      p.x_ptiles = static_cast<int>(ptiles);
      p.x_ctiles = static_cast<int>(ctiles);
    }
  }
  if (p.fused) {
    const int KC = block_elems_of(prec);
    const int nA = prec == PREC_F32 ? 2 : 1, nB = nA;
    p.CBg = static_cast<int>(cdiv(p.Cg, KC));
    const int64_t numKB = int64_t(p.dg) * p.T * p.CBg;
    const int max_rows = prec == PREC_F32 ? 256 : 512;
    p.cchunks = static_cast<int>(cdiv(p.O, max_rows));
    const int rows_per_chunk = static_cast<int>(cdiv(p.O, p.cchunks));
    p.nsub = static_cast<int>(cdiv(rows_per_chunk, 256));
    p.n_mma = static_cast<int>(cdiv(cdiv(rows_per_chunk, p.nsub), 16) * 16);
    p.nrows = p.nsub * p.n_mma;
    p.acc_bufs = (2 * p.nrows <= 512) ? 2 : 1;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(p.acc_bufs * p.nrows)) cols <<= 1;
    p.tmem_cols = cols;
    // fp16 / int8 tiles of this kernel run as CTA pairs (M = 256 per MMA, each CTA holding half
    // of B) when they carry more than 256 output channels: each CTA then copies half of the
    // 512-row weight tile per K-block, and four stages fit instead of two (512-channel dg8
    // layer: fp16 2.29 -> 2.20 ms, int8 2.31 -> 1.99 ms). Up to 256 channels one CTA per tile
    // measured faster (the pair adds a cross-CTA hand-off to every K-block); the TMEM-A kernel,
    // which takes those layers, has no pair variant (measured 0.43-0.46 against 0.35 ms). The
    // override forces either here.
    const int pov = g_pair_override.load();
    p.pair = (prec == PREC_F16 || prec == PREC_I8) &&
             (pov == POV_PAIRS || (pov == POV_AUTO && p.nsub >= 2));
    p.a_stage_bytes = static_cast<uint32_t>(nA * kATileBytes);
    p.b_kb_bytes = size_t(nB) * p.nrows * kRowBytes;
    p.b_stage_bytes = static_cast<uint32_t>(p.b_kb_bytes / (p.pair ? 2 : 1));
    const size_t per_stage = p.a_stage_bytes + p.b_stage_bytes;
    // alignment slack + barriers and flags + the staged bias of one output-channel chunk
    const size_t fixed = 1024 + 512 + size_t(p.nrows) * sizeof(float);
    int stages = static_cast<int>((kSmemLimit - fixed) / per_stage);
    if (stages > kMaxStages) stages = kMaxStages;
    const int64_t cta_tiles_per_img = cdiv(P, kTileM);
    const int64_t tiles_per_img = p.pair ? cdiv(P, 2 * kTileM) : cta_tiles_per_img;
    const int64_t num_tiles = int64_t(p.N) * tiles_per_img * p.cchunks;
    if (stages < 2 || numKB >= (int64_t(1) << 31) || num_tiles >= (int64_t(1) << 31)) {
      p.fused = false;
    } else {
      p.stages = stages;
      p.numKB = static_cast<int>(numKB);
      p.tiles_per_img = static_cast<int>(tiles_per_img);
      p.num_tiles = static_cast<int>(num_tiles);
      p.smem_bytes = fixed + size_t(stages) * per_stage;
      // Window of x: whole rows (W <= 256, one TMA box) covering every tap of every pixel of a
      // CTA's 128 pixels whose offsets lie in (-1 - M, 1 + M), for the largest margin M <= 2
      // that still leaves three pipeline stages (else two). Corners outside it are read from
      // global memory.
      if (p.W <= 256) {
        int rows_max = 0;
        const int64_t loop = cta_tiles_per_img < 4096 ? cta_tiles_per_img : 4096;
        for (int64_t pt = 0; pt < loop; ++pt) {
          const int64_t a0 = pt * kTileM, a1 = (a0 + kTileM < P ? a0 + kTileM : P) - 1;
          const int rows = static_cast<int>(a1 / p.Wo - a0 / p.Wo + 1);
          if (rows > rows_max) rows_max = rows;
        }
        if (cta_tiles_per_img > 4096 && p.Wo > 4096) rows_max = 1 << 20;  // no exact bound
        const int64_t base = int64_t(rows_max - 1) * p.stride + int64_t(p.K - 1) * p.dil + 3;
        bool done = false;
        for (int want = 3; want >= 2 && !done; --want) {
          for (int M = 2; M >= 0; --M) {
            const int64_t rows = base + 2 * M;
            if (rows > 256) continue;
            const size_t wb = size_t(rows) * p.W * kRowBytes;
            // window byte offsets travel in 16 bits
            if (wb > 65536 || 2 * wb + fixed + size_t(want) * per_stage > kSmemLimit) continue;
            int sw = static_cast<int>((kSmemLimit - fixed - 2 * wb) / per_stage);
            if (sw > kMaxStages) sw = kMaxStages;
            p.use_win = true;
            p.win_rows = static_cast<int>(rows);
            p.win_top = p.pad + 1 + M;
            p.win_bytes = static_cast<uint32_t>(wb);
            p.stages = sw;
            p.smem_bytes = fixed + size_t(sw) * per_stage + 2 * wb;
            done = true;
            break;
          }
        }
      }
      // fp32 outputs (int8, TF32) leave the epilogue through TMA stores: two [16 channels]
      // [32 pixels] staging boxes per epilogue warp after the staged bias, when they fit beside
      // the stages chosen above and y's rows (P elements) are whole multiples of 16 bytes
      // (tensor-map strides). 512-channel dg8 layer, int8: 1.297 -> 1.232 ms. fp16 keeps its
      // direct paired stores (its 1 KB boxes measured 2 % slower: 1.913 -> 1.95 ms).
      const size_t y_eb = 4;
      const size_t epi_bytes = size_t(kNumEpiWarps) * 2 * 16 * 32 * y_eb;
      if (prec != PREC_F16 && (size_t(P) * y_eb) % 16 == 0 &&
          p.smem_bytes + epi_bytes + 128 <= kSmemLimit) {
        p.epi_off = static_cast<uint32_t>(512 + cdiv(int64_t(p.nrows) * 4, 128) * 128);
        p.smem_bytes += epi_bytes + 128;
      }
    }
  }
  // fp16 / int8 with at most 256 output channels take the kernel with the A operand in TMEM
  // (override "smem" keeps the shared-memory A kernel; "ta" also uses it for wider layers, one
  // output-channel chunk of <= 256 per tile).
  if (p.fused && (prec == PREC_F16 || prec == PREC_I8)) {
    const int kov = g_kernel_override.load();
    const bool force_smem = kov == KOV_SMEM;
    const bool force_ta = kov == KOV_TA;
    if (!force_smem && (p.O <= 256 || force_ta)) {
      Plan t = p;
      t.pair = false;  // the TMEM-A kernel runs one CTA per tile
      plan_ta(&t);
      if (t.ta) p = t;
    }
  }
  // int8 3x3 layers of the A-in-shared-memory kernel whose groups hold 64 channels (half of the
  // 128-byte int8 K-block) and that run without a window: two taps per K-block (channels of tap
  // 2i in bytes 0-63, of tap 2i+1 in bytes 64-127), 5 K-blocks per group instead of 9 half-empty
  // ones.
  if (p.fused && !p.ta && prec == PREC_I8 && !p.use_win && p.T == 9 && p.Cg == 64) {
    p.tap_pairs = true;
    p.numKB = p.dg * ((p.T + 1) / 2);
  }
  // Workspace: [error word | x channels-last | packed weights]; +256 so that any base pointer
  // can be aligned up to 256 bytes.
  if (p.fused) p.kind = KIND_TCGEN05;
  size_t off = kErrBytes;
  if (p.kind == KIND_TCGEN05) {
    p.off_x = off;
    off = align_up(off + size_t(p.N) * plane * p.elem_bytes, 1024);
    p.off_w = off;
    off += size_t(p.cchunks) * p.numKB * p.b_kb_bytes;
  } else if (p.kind == KIND_F32_EXACT) {
    p.off_x = off;
    off = align_up(off + size_t(p.N) * plane * sizeof(float), 1024);
    p.off_w = off;
    off += size_t(p.x_ctiles) * p.numKB * kXK * kXCo * sizeof(float);
  }
  p.ws_bytes = align_up(off, 256) + 256;
  return DCNV2_OK;
}

using FusedFn = void (*)(const FusedArgs, const CUtensorMap);
using FusedFnY = void (*)(const FusedArgs, const CUtensorMap, const CUtensorMap);

template <typename F>
bool set_smem_attr(F* kfn) {
  return cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSmemLimit)) == cudaSuccess;
}

// Launch configuration of a main kernel: programmatic stream serialization (it may start while
// the kernel ahead of it in the stream finishes, and calls griddep_wait before reading that
// kernel's outputs) and, for `pair`, clusters of 2 CTAs along x. The attributes are written into
// the caller's `attr`, which must outlive the launch call.
cudaLaunchConfig_t main_launch_config(int grid, int threads, size_t smem, cudaStream_t st,
                                      cudaLaunchAttribute (&attr)[2], bool pair) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pair ? 2 : 1;
  return cfg;
}

// The offset / mask head of dcnv2_forward_with_head: its packed weights, launch shape and
// tensor map, launched by launch_fused between the layer's pre-passes and its main kernel.
struct HeadLaunch {
  HeadArgs a;
  const void* weight = nullptr;  // [n_head][C][K][K] fp16
  int cb = 0;                    // channel blocks of 64
  size_t smem = 0;
  int grid = 0;
};

dcnv2_status launch_head_pack(const HeadLaunch& h, DevInfo* di, cudaStream_t st, Marks& mk) {
  const size_t total = size_t(h.a.numKB) * h.a.n_mma * 8;
  int64_t blocks = cdiv(static_cast<int64_t>(total), 256);
  const int64_t cap = int64_t(di->sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  mk.mark(st);
  pack_weights_kernel<PREC_F16><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      h.weight, const_cast<uint8_t*>(h.a.wpack), h.a.err, h.a.n_head, h.a.C, h.a.T, h.a.C, h.cb,
      h.a.numKB, h.a.n_mma, 1, 0, 0);
  return cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
}

dcnv2_status launch_head(const HeadLaunch& h, DevInfo* di, const void* x_nhwc, cudaStream_t st,
                         Marks& mk) {
  constexpr uint32_t kHeadBit = 1u << 5;
  if (!(di->attr_set.load(std::memory_order_acquire) & kHeadBit)) {
    if (!set_smem_attr(dcnv2_offset_head_kernel)) {
      cudaGetLastError();
      return DCNV2_ERR_CUDA;
    }
    di->attr_set.fetch_or(kHeadBit, std::memory_order_acq_rel);
  }
  // channels-last x as bytes {C*2, W, H, N}; box = one 128-byte channel block of TR rows x TW
  // columns, 128-byte swizzle (the MMA's A tile layout)
  const HeadArgs& a = h.a;
  const cuuint64_t dims[4] = {cuuint64_t(a.C) * 2, cuuint64_t(a.W), cuuint64_t(a.H),
                              cuuint64_t(a.N)};
  const cuuint64_t strides[3] = {cuuint64_t(a.C) * 2, cuuint64_t(a.W) * a.C * 2,
                                 cuuint64_t(a.H) * a.W * a.C * 2};
  const cuuint32_t rows = static_cast<cuuint32_t>(a.win_mode ? a.TR + a.K - 1 : a.TR);
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(kRowBytes), static_cast<cuuint32_t>(a.TW),
                             rows, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUtensorMap tmap;
  std::memset(&tmap, 0, sizeof(tmap));
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode || encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(x_nhwc), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DCNV2_ERR_CUDA;
  mk.mark(st);
  cudaLaunchAttribute at[2];
  const cudaLaunchConfig_t cfg = main_launch_config(h.grid, kHeadThreads, h.smem, st, at, false);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, dcnv2_offset_head_kernel, a, tmap);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
}

template <int PREC>
dcnv2_status launch_fused(const Plan& p, DevInfo* di, int dev, const void* x, const void* offset,
                          const void* mask, const void* weight, const void* bias, void* y,
                          uint8_t* ws, float scale, cudaStream_t st, Marks& mk,
                          const HeadLaunch* head = nullptr) {
  using TR = PrecTraits<PREC>;
  using XT = typename TR::X;
  constexpr bool kCanPair = PREC == PREC_F16 || PREC == PREC_I8;
  const uint32_t bit = 1u << PREC;
  if (!(di->attr_set.load(std::memory_order_acquire) & bit)) {
    bool ok = set_smem_attr(dcnv2_fused_kernel<PREC, false, 9, false>) &&
              set_smem_attr(dcnv2_fused_kernel<PREC, false, 0, false>);
    if constexpr (kCanPair)
      ok = ok && set_smem_attr(dcnv2_fused_kernel<PREC, false, 9, true>) &&
           set_smem_attr(dcnv2_fused_kernel<PREC, false, 0, true>);
    if constexpr (PREC == PREC_F16)
      ok = ok && set_smem_attr(dcnv2_fused_kernel<PREC, true, 9, false>) &&
           set_smem_attr(dcnv2_fused_kernel<PREC, true, 0, false>) &&
           set_smem_attr(dcnv2_fused_kernel<PREC, true, 9, true>) &&
           set_smem_attr(dcnv2_fused_kernel<PREC, true, 0, true>) &&
           set_smem_attr(dcnv2_fused_ta_kernel<PREC, false, 9>) &&
           set_smem_attr(dcnv2_fused_ta_kernel<PREC, false, 0>) &&
           set_smem_attr(dcnv2_fused_ta_kernel<PREC, true, 0>) &&
           set_smem_attr(dcnv2_fused_ta_kernel<PREC, true, 9>);
    if constexpr (PREC == PREC_I8)
      ok = ok && set_smem_attr(dcnv2_fused_ta_kernel<PREC, false, 0>) &&
           set_smem_attr(dcnv2_fused_ta_kernel<PREC, false, 9>);
    if (!ok) return DCNV2_ERR_CUDA;
    di->attr_set.fetch_or(bit, std::memory_order_acq_rel);
  }
  (void)dev;
  int* err = reinterpret_cast<int*>(ws);
  XT* x_nhwc = reinterpret_cast<XT*>(ws + p.off_x);
  uint8_t* wpack = ws + p.off_w;

  // 1) one launch: x NCHW -> channels-last (tiled kernels where the channel and pixel counts
  // allow, the generic tile otherwise) and the weights -> swizzled B tiles (also clears the
  // error word)
  {
    const int HW = p.H * p.W;
    const bool aligned16 = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                           (reinterpret_cast<uintptr_t>(x_nhwc) & 15u) == 0;
    const bool tiled = aligned16 && HW % 128 == 0 &&
                       ((PREC == PREC_F16 && p.C % 64 == 0) || (PREC == PREC_I8 && p.C % 128 == 0));
    PrepassArgs pa;
    pa.x = x; pa.xt = x_nhwc; pa.C = p.C; pa.HW = HW; pa.tiled = tiled ? 1 : 0;
    if (tiled) {
      pa.tiles_x = HW / 128;
      pa.tiles_y = p.C / (PREC == PREC_F16 ? 64 : 128);
    } else {
      constexpr int TILE = 8 * (16 / static_cast<int>(sizeof(XT)));
      pa.tiles_x = static_cast<int>(cdiv(HW, TILE));
      pa.tiles_y = static_cast<int>(cdiv(p.C, TILE));
    }
    const int64_t tr_blocks = int64_t(pa.tiles_x) * pa.tiles_y * p.N;
    const size_t total = size_t(p.cchunks) * p.numKB * p.nrows * 8;
    int64_t pk_blocks = cdiv(static_cast<int64_t>(total), 256);
    const int64_t cap = int64_t(di->sm_count) * 8;
    if (pk_blocks > cap) pk_blocks = cap;
    if (pk_blocks < 1) pk_blocks = 1;
    if (tr_blocks + pk_blocks >= (int64_t(1) << 31)) return DCNV2_ERR_INVALID_ARG;
    pa.tr_blocks = static_cast<int>(tr_blocks);
    pa.w = weight; pa.wpack = wpack; pa.err = err;
    pa.O = p.O; pa.T = p.T; pa.Cg = p.Cg; pa.CBg = p.CBg; pa.numKB = p.numKB;
    pa.nrows = p.nrows; pa.cchunks = p.cchunks; pa.half_mma = p.pair ? p.n_mma / 2 : 0;
    pa.tap_pairs = p.tap_pairs ? 1 : 0;
    mk.mark(st);
    prepass_kernel<PREC><<<static_cast<unsigned>(tr_blocks + pk_blocks), 256, 0, st>>>(pa);
  }
  // 1b) the offset / mask head's weights (also clears the error word)
  if (head) {
    const dcnv2_status hs = launch_head_pack(*head, di, st, mk);
    if (hs != DCNV2_OK) return hs;
  }
  // 2b) the offset / mask head from the channels-last x; the main kernel reads its outputs
  if (head) {
    const dcnv2_status hs = launch_head(*head, di, x_nhwc, st, mk);
    if (hs != DCNV2_OK) return hs;
  }
  // 3) the fused implicit GEMM
  FusedArgs a;
  a.x_nhwc = reinterpret_cast<const uint8_t*>(x_nhwc);
  a.offset = offset; a.mask = mask; a.wpack = wpack; a.bias = bias; a.y = y; a.err = err;
  a.N = p.N; a.C = p.C; a.H = p.H; a.W = p.W; a.O = p.O; a.Ho = p.Ho; a.Wo = p.Wo; a.P = p.P;
  a.K = p.K; a.T = p.T; a.stride = p.stride; a.pad = p.pad; a.dil = p.dil; a.dg = p.dg;
  a.Cg = p.Cg; a.CBg = p.CBg; a.numKB = p.numKB;
  a.tiles_per_img = p.tiles_per_img; a.cchunks = p.cchunks; a.num_tiles = p.num_tiles;
  a.n_mma = p.n_mma; a.nsub = p.nsub; a.nrows = p.nrows; a.acc_bufs = p.acc_bufs;
  a.stages = p.stages; a.tmem_cols = p.tmem_cols;
  a.a_stage_bytes = p.a_stage_bytes; a.b_stage_bytes = p.b_stage_bytes;
  a.scale = scale; a.precise = p.precise ? 1 : 0; a.tf32_single = p.tf32_single ? 1 : 0;
  a.timeout_ns = kDefaultTimeoutNs;
  a.use_win = 0; a.win_rows = p.win_rows; a.win_top = p.win_top; a.win_bytes = p.win_bytes;
  a.win_stride = p.win_stride; a.a_stages = p.a_stages; a.b_stages = p.b_stages;
  a.tap_pairs = p.tap_pairs ? 1 : 0;
  // y as a [N][O][P] tensor for the epilogue's TMA stores (boxes of 32 pixels x 16 channels);
  // without a map the epilogue stores y directly
  a.epi_off = 0;
  CUtensorMap tmap_y;
  std::memset(&tmap_y, 0, sizeof(tmap_y));
  if (PREC != PREC_F16 && p.epi_off != 0 && !p.ta && (reinterpret_cast<uintptr_t>(y) % 16) == 0) {
    const cuuint64_t eb = 4;
    const cuuint64_t dims[3] = {cuuint64_t(p.P), cuuint64_t(p.O), cuuint64_t(p.N)};
    const cuuint64_t strides[2] = {cuuint64_t(p.P) * eb, cuuint64_t(p.O) * p.P * eb};
    const cuuint32_t box[3] = {32u, 16u, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode && encode(&tmap_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, y, dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      a.epi_off = p.epi_off;
  }
  CUtensorMap tmap;
  std::memset(&tmap, 0, sizeof(tmap));
  if (p.use_win) {
    // x channels-last seen as bytes: dims {C*EB, W, H, N}; box = one 128-byte channel block of
    // win_rows whole rows of one image.
    const cuuint64_t eb = static_cast<cuuint64_t>(p.elem_bytes);
    const cuuint64_t dims[4] = {cuuint64_t(p.C) * eb, cuuint64_t(p.W), cuuint64_t(p.H),
                                cuuint64_t(p.N)};
    const cuuint64_t strides[3] = {cuuint64_t(p.C) * eb, cuuint64_t(p.W) * p.C * eb,
                                   cuuint64_t(p.H) * p.W * p.C * eb};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(kRowBytes), static_cast<cuuint32_t>(p.W),
                               static_cast<cuuint32_t>(p.win_rows), 1u};
    const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode && encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, x_nhwc, dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      a.use_win = 1;  // otherwise every corner is read from global memory
  }
  mk.mark(st);
  // 3x3 kernels take the variant with the nine taps unrolled
  const bool k3 = p.T == 9;
  cudaError_t e = cudaSuccess;
  if constexpr (kCanPair) {
    if (p.ta) {
      FusedFn kfn;
      if constexpr (PREC == PREC_F16) {
        if (p.precise && k3) kfn = dcnv2_fused_ta_kernel<PREC, true, 9>;
        else if (p.precise) kfn = dcnv2_fused_ta_kernel<PREC, true, 0>;
        else if (k3) kfn = dcnv2_fused_ta_kernel<PREC, false, 9>;
        else kfn = dcnv2_fused_ta_kernel<PREC, false, 0>;
      } else {
        kfn = k3 ? dcnv2_fused_ta_kernel<PREC, false, 9> : dcnv2_fused_ta_kernel<PREC, false, 0>;
      }
      const int grid = p.num_tiles < di->sm_count ? p.num_tiles : di->sm_count;
      cudaLaunchAttribute at[2];
      const cudaLaunchConfig_t cfg = main_launch_config(grid, kTaThreads, p.smem_bytes, st, at,
                                                        false);
      e = cudaLaunchKernelEx(&cfg, kfn, a, tmap);
      mk.mark(st);
      return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
    }
    if (p.pair) {
      FusedFnY kfn = k3 ? dcnv2_fused_kernel<PREC, false, 9, true>
                        : dcnv2_fused_kernel<PREC, false, 0, true>;
      if constexpr (PREC == PREC_F16) {
        if (p.precise)
          kfn = k3 ? dcnv2_fused_kernel<PREC, true, 9, true> : dcnv2_fused_kernel<PREC, true, 0, true>;
      }
      int clusters = di->pair_clusters[PREC].load(std::memory_order_acquire);
      if (clusters <= 0) {
        // co-resident CTA pairs of this kernel (one CTA per SM); a persistent grid of that size
        cudaLaunchAttribute qa[2];
        cudaLaunchConfig_t qc = main_launch_config(1, kThreads, p.smem_bytes, st, qa, true);
        if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &qc) != cudaSuccess || clusters < 1) {
          cudaGetLastError();
          clusters = di->sm_count / 2;
        }
        di->pair_clusters[PREC].store(clusters, std::memory_order_release);
      }
      const int nc = p.num_tiles < clusters ? p.num_tiles : clusters;
      cudaLaunchAttribute at[2];
      cudaLaunchConfig_t cfg = main_launch_config(2 * nc, kThreads, p.smem_bytes, st, at, true);
      e = cudaLaunchKernelEx(&cfg, kfn, a, tmap, tmap_y);
      mk.mark(st);
      return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
    }
  }
  const int grid = p.num_tiles < di->sm_count ? p.num_tiles : di->sm_count;
  FusedFnY kfn = k3 ? dcnv2_fused_kernel<PREC, false, 9, false>
                    : dcnv2_fused_kernel<PREC, false, 0, false>;
  if constexpr (PREC == PREC_F16) {
    if (p.precise)
      kfn = k3 ? dcnv2_fused_kernel<PREC, true, 9, false> : dcnv2_fused_kernel<PREC, true, 0, false>;
  }
  cudaLaunchAttribute at[2];
  const cudaLaunchConfig_t cfg = main_launch_config(grid, kThreads, p.smem_bytes, st, at, false);
  e = cudaLaunchKernelEx(&cfg, kfn, a, tmap, tmap_y);
  mk.mark(st);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
}

dcnv2_status launch_f32_exact(const Plan& p, DevInfo* di, const void* x, const void* offset,
                              const void* mask, const void* weight, const void* bias, void* y,
                              uint8_t* ws, cudaStream_t st, Marks& mk) {
  int* err = reinterpret_cast<int*>(ws);
  float* x_nhwc = reinterpret_cast<float*>(ws + p.off_x);
  float* wplain = reinterpret_cast<float*>(ws + p.off_w);
  // one pre-pass launch: transpose (32 x 32 tiles) and k-major weight packing
  {
    const int HW = p.H * p.W;
    PrepassPlainArgs pa;
    pa.x = reinterpret_cast<const float*>(x); pa.xt = x_nhwc; pa.C = p.C; pa.HW = HW;
    pa.tiles_x = static_cast<int>(cdiv(HW, 32));
    pa.tiles_y = static_cast<int>(cdiv(p.C, 32));
    const int64_t tr_blocks = int64_t(pa.tiles_x) * pa.tiles_y * p.N;
    const size_t total = size_t(p.x_ctiles) * p.numKB * kXK * kXCo;
    int64_t pk_blocks = cdiv(static_cast<int64_t>(total), 256);
    const int64_t cap = int64_t(di->sm_count) * 8;
    if (pk_blocks > cap) pk_blocks = cap;
    if (pk_blocks < 1) pk_blocks = 1;
    if (tr_blocks + pk_blocks >= (int64_t(1) << 31)) return DCNV2_ERR_INVALID_ARG;
    pa.tr_blocks = static_cast<int>(tr_blocks);
    pa.w = reinterpret_cast<const float*>(weight); pa.wp = wplain; pa.err = err;
    pa.O = p.O; pa.T = p.T; pa.Cg = p.Cg; pa.CBg = p.CBg; pa.numKB = p.numKB;
    pa.ctiles = p.x_ctiles;
    mk.mark(st);
    prepass_plain_kernel<<<static_cast<unsigned>(tr_blocks + pk_blocks), 256, 0, st>>>(pa);
  }
  ExactArgs a;
  a.x_nhwc = x_nhwc; a.offset = reinterpret_cast<const float*>(offset);
  a.mask = reinterpret_cast<const float*>(mask); a.wplain = wplain;
  a.bias = reinterpret_cast<const float*>(bias); a.y = reinterpret_cast<float*>(y);
  a.N = p.N; a.C = p.C; a.H = p.H; a.W = p.W; a.O = p.O; a.Ho = p.Ho; a.Wo = p.Wo; a.P = p.P;
  a.K = p.K; a.T = p.T; a.stride = p.stride; a.pad = p.pad; a.dil = p.dil; a.dg = p.dg;
  a.Cg = p.Cg; a.CBg = p.CBg; a.numKB = p.numKB; a.ptiles = p.x_ptiles; a.ctiles = p.x_ctiles;
  const int64_t grid = int64_t(p.N) * p.x_ptiles * p.x_ctiles;
  constexpr uint32_t kExactBit = 1u << 4;
  if (!(di->attr_set.load(std::memory_order_acquire) & kExactBit)) {
    if (cudaFuncSetAttribute(dcnv2_f32_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kXSmemBytes)) != cudaSuccess) {
      cudaGetLastError();
      return DCNV2_ERR_CUDA;
    }
    di->attr_set.fetch_or(kExactBit, std::memory_order_acq_rel);
  }
  mk.mark(st);
  cudaLaunchAttribute at[2];
  const cudaLaunchConfig_t cfg = main_launch_config(static_cast<int>(grid), kXThreads * kXGroups,
                                                    kXSmemBytes, st, at, false);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, dcnv2_f32_exact_kernel, a);
  mk.mark(st);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
}

template <int PREC>
dcnv2_status launch_simt(const Plan& p, DevInfo* di, const void* x, const void* offset,
                         const void* mask, const void* weight, const void* bias, void* y,
                         uint8_t* ws, float scale, cudaStream_t st, Marks& mk) {
  if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return DCNV2_ERR_CUDA;
  SimtArgs a;
  a.x = x; a.offset = offset; a.mask = mask; a.w = weight; a.bias = bias; a.y = y;
  a.N = p.N; a.C = p.C; a.H = p.H; a.W = p.W; a.O = p.O; a.Ho = p.Ho; a.Wo = p.Wo; a.P = p.P;
  a.K = p.K; a.T = p.T; a.stride = p.stride; a.pad = p.pad; a.dil = p.dil; a.dg = p.dg;
  a.Cg = p.Cg; a.scale = scale; a.i8_rint = p.i8_rint ? 1 : 0;
  const size_t total = size_t(p.N) * p.O * p.P;
  int64_t blocks = cdiv(static_cast<int64_t>(total), 256);
  const int64_t cap = int64_t(di->sm_count) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  mk.mark(st);
  dcnv2_simt_kernel<PREC><<<static_cast<unsigned>(blocks), 256, 0, st>>>(a);
  mk.mark(st);
  return cudaGetLastError() == cudaSuccess ? DCNV2_OK : DCNV2_ERR_CUDA;
}

bool aligned(const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

// ---- failure-detection self test: a wait that nothing completes ----
__global__ void selftest_timeout_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_addr(&bar), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const WaitCtx wc{timeout_ns, err, &abort_flag};
  if (threadIdx.x == 0) {
    // Parity 0 of a fresh barrier completes only after one arrival, which never comes.
    if (!wait_bar(ptx::smem_addr(&bar), 0, wc, DCNV2_DEVERR_TIMEOUT_MMA)) {
      // the error bit is already set by wait_bar
    }
    // Complete the phase so that the barrier is left in a clean state.
    ptx::mbar_arrive(ptx::smem_addr(&bar));
  }
  __syncthreads();
}

}  // namespace
}  // namespace dcnv2

using namespace dcnv2;

extern "C" {

dcnv2_status dcnv2_output_shape(const dcnv2_desc* desc, int64_t out_dims[4]) {
  if (!out_dims) return DCNV2_ERR_INVALID_ARG;
  Plan p;
  const dcnv2_status s = make_plan(desc, &p);
  if (s != DCNV2_OK) return s;
  out_dims[0] = p.N; out_dims[1] = p.O; out_dims[2] = p.Ho; out_dims[3] = p.Wo;
  return DCNV2_OK;
}

size_t dcnv2_workspace_size(const dcnv2_desc* desc) {
  Plan p;
  if (make_plan(desc, &p) != DCNV2_OK) return 0;
  return p.ws_bytes;
}

int32_t dcnv2_uses_tensor_cores(const dcnv2_desc* desc) {
  Plan p;
  if (make_plan(desc, &p) != DCNV2_OK) return 0;
  return p.kind;
}

const char* dcnv2_diag_main_kernel(const dcnv2_desc* desc) {
  Plan p;
  if (make_plan(desc, &p) != DCNV2_OK) return nullptr;
  switch (p.kind) {
    case KIND_TCGEN05: return p.ta ? "dcnv2_fused_ta_kernel" : "dcnv2_fused_kernel";
    case KIND_F32_EXACT: return "dcnv2_f32_exact_kernel";
    default: return "dcnv2_simt_kernel";
  }
}

int32_t dcnv2_launch_count(const dcnv2_desc* desc) {
  Plan p;
  if (make_plan(desc, &p) != DCNV2_OK) return 0;
  if (p.kind == KIND_SIMT) return 1;
  return 2;  // pre-pass (transpose + weight packing), main kernel
}

static dcnv2_status forward_impl(const dcnv2_desc* desc, const void* x, const void* offset,
                                 const void* mask, const void* weight, const void* bias, void* y,
                                 void* workspace, size_t workspace_bytes, float x_scale,
                                 float w_scale, dcnv2_stream_t stream, Marks& mk) {
  Plan p;
  dcnv2_status s = make_plan(desc, &p);
  if (s != DCNV2_OK) return s;
  if (!x || !offset || !mask || !weight || !y) return DCNV2_ERR_INVALID_ARG;
  const size_t eb = static_cast<size_t>(p.elem_bytes);
  const size_t gb = p.prec == PREC_F16 ? 2 : 4;  // offset / mask / bias / y elements
  if (!aligned(x, eb) || !aligned(weight, eb) || !aligned(offset, gb) || !aligned(mask, gb) ||
      !aligned(y, gb) || (bias && !aligned(bias, gb)))
    return DCNV2_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < p.ws_bytes) return DCNV2_ERR_WORKSPACE;
  float scale = 1.f;
  if (p.prec == PREC_I8) {
    if (!(x_scale > 0.f) || !(w_scale > 0.f) || !std::isfinite(x_scale) || !std::isfinite(w_scale))
      return DCNV2_ERR_INVALID_ARG;
    scale = x_scale * w_scale;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return DCNV2_ERR_NO_DEVICE; }
  DevInfo* di = device_info(dev);
  if (!di || !di->ok) return DCNV2_ERR_NO_DEVICE;
  if (di->major != 10) return DCNV2_ERR_NO_DEVICE;  // built for sm_100a only
  uint8_t* ws = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(workspace), 256));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.kind == KIND_F32_EXACT)
    return launch_f32_exact(p, di, x, offset, mask, weight, bias, y, ws, st, mk);
  if (p.fused) {
    switch (p.prec) {
      case PREC_F16: return launch_fused<PREC_F16>(p, di, dev, x, offset, mask, weight, bias, y, ws, scale, st, mk);
      case PREC_I8: return launch_fused<PREC_I8>(p, di, dev, x, offset, mask, weight, bias, y, ws, scale, st, mk);
      default: return launch_fused<PREC_F32>(p, di, dev, x, offset, mask, weight, bias, y, ws, scale, st, mk);
    }
  }
  switch (p.prec) {
    case PREC_F16: return launch_simt<PREC_F16>(p, di, x, offset, mask, weight, bias, y, ws, scale, st, mk);
    case PREC_I8: return launch_simt<PREC_I8>(p, di, x, offset, mask, weight, bias, y, ws, scale, st, mk);
    default: return launch_simt<PREC_F32>(p, di, x, offset, mask, weight, bias, y, ws, scale, st, mk);
  }
}

dcnv2_status dcnv2_forward(const dcnv2_desc* desc, const void* x, const void* offset,
                           const void* mask, const void* weight, const void* bias, void* y,
                           void* workspace, size_t workspace_bytes, float x_scale, float w_scale,
                           dcnv2_stream_t stream) {
  Marks none;
  return forward_impl(desc, x, offset, mask, weight, bias, y, workspace, workspace_bytes, x_scale,
                      w_scale, stream, none);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Layer with its offset / mask head: om = Conv2d(C -> 3*dg*K*K, K, stride 1, padding (K-1)/2)(x)
// on tensor cores from the layer's own channels-last copy of x, offset = om[:, :2*dg*K*K],
// mask = sigmoid(om[:, 2*dg*K*K:]), then the deformable layer on them.
namespace {

struct HeadPlan {
  Plan p;
  HeadLaunch h;
  size_t off_hw = 0, off_off = 0, off_msk = 0, total = 0;  // from the 256-aligned base
};

dcnv2_status make_head_plan(const dcnv2_desc* d, HeadPlan* hp) {
  const dcnv2_status st = make_plan(d, &hp->p);
  if (st != DCNV2_OK) return st;
  const Plan& p = hp->p;
  // fp16 layers on the tensor-core path; the head is a stride-1, dilation-1 "same" convolution,
  // so the layer must have the same output size (stride 1, dilation 1, padding (K-1)/2)
  if (p.prec != PREC_F16 || p.kind != KIND_TCGEN05) return DCNV2_ERR_UNSUPPORTED;
  if (p.stride != 1 || p.dil != 1 || p.K % 2 == 0 || p.pad != (p.K - 1) / 2)
    return DCNV2_ERR_UNSUPPORTED;
  if (p.C % 8 != 0) return DCNV2_ERR_UNSUPPORTED;  // 16-byte rows of the channels-last copy
  const int n_head = 3 * p.dg * p.T;
  if (n_head > 256) return DCNV2_ERR_UNSUPPORTED;  // one MMA of N <= 256
  HeadArgs& a = hp->h.a;
  a = HeadArgs{};
  a.N = p.N; a.C = p.C; a.H = p.H; a.W = p.W; a.K = p.K; a.pad = p.pad; a.T = p.T;
  a.n_head = n_head;
  a.n_off = 2 * p.dg * p.T;
  a.n_mma = static_cast<int>(cdiv(n_head, 16) * 16);
  hp->h.cb = static_cast<int>(cdiv(p.C, 64));
  a.numKB = hp->h.cb * p.T;
  // Window mode where the tile's columns are a multiple of 8 and two stages (a channel block's
  // K windows + its K*K weight tiles each) fit: tiles of 8 x 16 pixels (16 x 8 below 16 columns);
  // otherwise one box per tap with the tile as wide as the image (up to 128 columns).
  const size_t fixed = 1024 + 256;  // alignment slack, barriers
  a.b_stage_bytes = static_cast<uint32_t>(a.n_mma) * kRowBytes;
  if (p.W >= 8) {
    const int tw = p.W >= 16 ? 16 : 8, tr = kTileM / tw;
    const uint32_t wb = static_cast<uint32_t>((tr + p.K - 1) * tw) * kRowBytes;
    const size_t stage = size_t(p.K) * wb + size_t(p.T) * a.b_stage_bytes;
    if (2 * stage + fixed <= kSmemLimit) {
      a.win_mode = 1;
      a.TW = tw;
      a.TR = tr;
      a.win_bytes = wb;
      a.stages = 2;
      hp->h.smem = fixed + 2 * stage;
    }
  }
  if (!a.win_mode) {
    int tw = 1;
    while (tw < p.W && tw < kTileM) tw <<= 1;
    a.TW = tw;
    a.TR = kTileM / tw;
    int stages = static_cast<int>((kSmemLimit - fixed) / (kHeadABytes + a.b_stage_bytes));
    a.stages = stages > kHeadMaxStages ? kHeadMaxStages : stages;
    hp->h.smem = fixed + size_t(a.stages) * (kHeadABytes + a.b_stage_bytes);
  }
  a.tiles_x = static_cast<int>(cdiv(p.W, a.TW));
  a.tiles_y = static_cast<int>(cdiv(p.H, a.TR));
  const int64_t tiles = int64_t(p.N) * a.tiles_x * a.tiles_y;
  if (tiles >= (int64_t(1) << 31)) return DCNV2_ERR_INVALID_ARG;
  a.num_tiles = static_cast<int>(tiles);
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(2 * a.n_mma)) cols <<= 1;
  a.tmem_cols = cols;
  a.timeout_ns = kDefaultTimeoutNs;
  const size_t plane = size_t(p.H) * p.W;
  size_t off = align_up(p.ws_bytes, 1024);
  hp->off_hw = off;
  off = align_up(off + size_t(a.numKB) * a.b_stage_bytes, 256);
  hp->off_off = off;
  off = align_up(off + size_t(p.N) * a.n_off * plane * 2, 256);
  hp->off_msk = off;
  off = align_up(off + size_t(p.N) * (n_head - a.n_off) * plane * 2, 256);
  hp->total = off + 256;
  return DCNV2_OK;
}

}  // namespace

extern "C" {

size_t dcnv2_forward_with_head_workspace_size(const dcnv2_desc* desc) {
  HeadPlan hp;
  return make_head_plan(desc, &hp) == DCNV2_OK ? hp.total : 0;
}

dcnv2_status dcnv2_forward_with_head(const dcnv2_desc* desc, const void* x,
                                     const void* head_weight, const void* head_bias,
                                     const void* weight, const void* bias, void* y,
                                     void* offset_out, void* mask_out, void* workspace,
                                     size_t workspace_bytes, dcnv2_stream_t stream) {
  HeadPlan hp;
  const dcnv2_status s = make_head_plan(desc, &hp);
  if (s != DCNV2_OK) return s;
  if (!x || !head_weight || !weight || !y) return DCNV2_ERR_INVALID_ARG;
  for (const void* ptr : {x, head_weight, head_bias, weight, bias, static_cast<const void*>(y),
                          static_cast<const void*>(offset_out), static_cast<const void*>(mask_out)})
    if (ptr && !aligned(ptr, 2)) return DCNV2_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < hp.total) return DCNV2_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return DCNV2_ERR_NO_DEVICE; }
  DevInfo* di = device_info(dev);
  if (!di || !di->ok || di->major != 10) return DCNV2_ERR_NO_DEVICE;
  uint8_t* ws = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(workspace), 256));
  HeadArgs& a = hp.h.a;
  a.wpack = ws + hp.off_hw;
  a.bias = static_cast<const __half*>(head_bias);
  a.offset = static_cast<__half*>(offset_out ? offset_out : ws + hp.off_off);
  a.mask = static_cast<__half*>(mask_out ? mask_out : ws + hp.off_msk);
  a.err = reinterpret_cast<int*>(ws);
  hp.h.weight = head_weight;
  hp.h.grid = a.num_tiles < di->sm_count ? a.num_tiles : di->sm_count;
  Marks none;
  return launch_fused<PREC_F16>(hp.p, di, dev, x, a.offset, a.mask, weight, bias, y, ws, 1.f,
                                reinterpret_cast<cudaStream_t>(stream), none, &hp.h);
}

dcnv2_status dcnv2_diag_forward_events(const dcnv2_desc* desc, const void* x, const void* offset,
                                       const void* mask, const void* weight, const void* bias,
                                       void* y, void* workspace, size_t workspace_bytes,
                                       float x_scale, float w_scale, dcnv2_stream_t stream,
                                       void* const* events, int32_t n_events) {
  const int32_t need = dcnv2_launch_count(desc) + 1;
  if (!events || n_events < need || need < 2) return DCNV2_ERR_INVALID_ARG;
  Marks mk;
  mk.ev = events;
  mk.n = n_events;
  return forward_impl(desc, x, offset, mask, weight, bias, y, workspace, workspace_bytes, x_scale,
                      w_scale, stream, mk);
}

dcnv2_status dcnv2_read_device_error(const void* workspace, dcnv2_stream_t stream,
                                     int32_t* code) {
  if (!workspace || !code) return DCNV2_ERR_INVALID_ARG;
  const uint8_t* ws =
      reinterpret_cast<const uint8_t*>(align_up(reinterpret_cast<uintptr_t>(workspace), 256));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, ws, sizeof(v), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    return DCNV2_ERR_CUDA;
  }
  *code = v;
  return v ? DCNV2_ERR_DEVICE_TIMEOUT : DCNV2_OK;
}

const char* dcnv2_status_string(dcnv2_status status) {
  switch (status) {
    case DCNV2_OK: return "ok";
    case DCNV2_ERR_INVALID_ARG: return "invalid argument";
    case DCNV2_ERR_UNSUPPORTED: return "unsupported dtype/format combination";
    case DCNV2_ERR_WORKSPACE: return "workspace missing or too small";
    case DCNV2_ERR_CUDA: return "CUDA runtime error";
    case DCNV2_ERR_NO_DEVICE: return "no sm_100 device";
    case DCNV2_ERR_DEVICE_TIMEOUT: return "kernel barrier wait timed out";
    case DCNV2_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the 32 MiB static buffer holds";
  }
  return "unknown status";
}

dcnv2_status dcnv2_diag_timeout_selftest(uint32_t timeout_us, int32_t* device_code) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return DCNV2_ERR_NO_DEVICE; }
  DevInfo* di = device_info(dev);
  if (!di || !di->ok || di->major != 10) return DCNV2_ERR_NO_DEVICE;
  int* err = nullptr;
  if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) { cudaGetLastError(); return DCNV2_ERR_CUDA; }
  dcnv2_status s = DCNV2_OK;
  int v = 0;
  if (cudaMemset(err, 0, sizeof(int)) != cudaSuccess) s = DCNV2_ERR_CUDA;
  if (s == DCNV2_OK) {
    selftest_timeout_kernel<<<1, 32>>>(err, 1000ull * timeout_us);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
      s = DCNV2_ERR_CUDA;
  }
  cudaFree(err);
  cudaGetLastError();
  if (device_code) *device_code = v;
  if (s != DCNV2_OK) return s;
  return v ? DCNV2_ERR_DEVICE_TIMEOUT : DCNV2_OK;
}

dcnv2_status dcnv2_diag_set_kernel_override(int32_t kernel, int32_t pair) {
  if (kernel < KOV_AUTO || kernel > KOV_SMEM || pair < POV_AUTO || pair > POV_SINGLE)
    return DCNV2_ERR_INVALID_ARG;
  read_env_overrides();  // the environment is read first, so it never undoes this call
  g_kernel_override.store(kernel);
  g_pair_override.store(pair);
  return DCNV2_OK;
}

dcnv2_status dcnv2_diag_binary_arch(int32_t* binary_version) {
  if (!binary_version) return DCNV2_ERR_INVALID_ARG;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, dcnv2_fused_ta_kernel<PREC_F16, false, 9>) != cudaSuccess) {
    cudaGetLastError();
    return DCNV2_ERR_NO_DEVICE;
  }
  *binary_version = fa.binaryVersion;
  return DCNV2_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Host-buffer forward: the batch in chunks of images, uploads / forwards / downloads overlapped.
namespace {

struct CopyStreams {
  cudaStream_t h2d = nullptr, d2h = nullptr;
  bool ok = false;
};
CopyStreams g_copy_streams[dcnv2::kMaxDevices];
std::once_flag g_copy_once[dcnv2::kMaxDevices];

// Two non-blocking copy streams per device, created once with that device current and kept for
// the life of the process (like the per-device launch attributes).
CopyStreams* copy_streams(int dev) {
  if (dev < 0 || dev >= dcnv2::kMaxDevices) return nullptr;
  std::call_once(g_copy_once[dev], [dev]() {
    CopyStreams& c = g_copy_streams[dev];
    c.ok = cudaStreamCreateWithFlags(&c.h2d, cudaStreamNonBlocking) == cudaSuccess &&
           cudaStreamCreateWithFlags(&c.d2h, cudaStreamNonBlocking) == cudaSuccess;
    if (!c.ok) cudaGetLastError();
  });
  return g_copy_streams[dev].ok ? &g_copy_streams[dev] : nullptr;
}

// Slots of the host-buffer forward: each holds x, offset, mask and y of one chunk, so that the
// upload of a chunk, the forward of the one before and the downloads of earlier ones overlap.
// Three or four slots measured the same as two (the bus, not the slot ring, sets the pace).
constexpr int kHostSlots = 2;

struct HostChunking {
  int chunk = 0;                        // images per chunk
  size_t x_img = 0, off_img = 0, mask_img = 0, y_img = 0;  // bytes per image
  size_t x_off = 0, off_off = 0, mask_off = 0, y_off = 0;  // slot offsets inside a slot block
  size_t slot_bytes = 0;                // one slot: x, offset, mask and y of a chunk
  size_t fwd_off = 0, fwd_bytes = 0;    // dcnv2_forward workspace of a full chunk
  size_t total = 0;
};

dcnv2_status host_chunking(const dcnv2_desc* desc, int32_t ipc, HostChunking* hc) {
  dcnv2::Plan full;
  const dcnv2_status s = dcnv2::make_plan(desc, &full);
  if (s != DCNV2_OK) return s;
  if (ipc < 0) return DCNV2_ERR_INVALID_ARG;
  int chunk = ipc > 0 ? ipc : (full.N + 7) / 8;
  if (chunk > full.N) chunk = full.N;
  if (chunk < 1) chunk = 1;
  dcnv2_desc d = *desc;
  d.n = chunk;
  dcnv2::Plan p;
  if (dcnv2::make_plan(&d, &p) != DCNV2_OK) return DCNV2_ERR_INVALID_ARG;
  const size_t eb = static_cast<size_t>(p.elem_bytes);
  const size_t gb = p.prec == dcnv2::PREC_F16 ? 2 : 4;  // offset / mask / y elements
  hc->chunk = chunk;
  hc->x_img = size_t(p.C) * p.H * p.W * eb;
  hc->off_img = size_t(2) * p.dg * p.T * p.P * gb;
  hc->mask_img = size_t(p.dg) * p.T * p.P * gb;
  hc->y_img = size_t(p.O) * p.P * gb;
  size_t off = 0;
  hc->x_off = off;    off = dcnv2::align_up(off + chunk * hc->x_img, 256);
  hc->off_off = off;  off = dcnv2::align_up(off + chunk * hc->off_img, 256);
  hc->mask_off = off; off = dcnv2::align_up(off + chunk * hc->mask_img, 256);
  hc->y_off = off;    off = dcnv2::align_up(off + chunk * hc->y_img, 256);
  hc->slot_bytes = off;
  hc->fwd_off = kHostSlots * off;
  hc->fwd_bytes = p.ws_bytes;
  hc->total = hc->fwd_off + p.ws_bytes + 256;
  return DCNV2_OK;
}

}  // namespace

extern "C" size_t dcnv2_forward_host_workspace_size(const dcnv2_desc* desc,
                                                    int32_t images_per_chunk) {
  HostChunking hc;
  return host_chunking(desc, images_per_chunk, &hc) == DCNV2_OK ? hc.total : 0;
}

extern "C" dcnv2_status dcnv2_forward_host(const dcnv2_desc* desc, const void* x_host,
                                           const void* offset_host, const void* mask_host,
                                           const void* weight, const void* bias, void* y_host,
                                           void* workspace, size_t workspace_bytes,
                                           float x_scale, float w_scale,
                                           int32_t images_per_chunk, dcnv2_stream_t stream) {
  HostChunking hc;
  dcnv2_status s = host_chunking(desc, images_per_chunk, &hc);
  if (s != DCNV2_OK) return s;
  if (!x_host || !offset_host || !mask_host || !weight || !y_host) return DCNV2_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < hc.total) return DCNV2_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return DCNV2_ERR_NO_DEVICE; }
  CopyStreams* cs = copy_streams(dev);
  if (!cs) return DCNV2_ERR_CUDA;
  uint8_t* ws = reinterpret_cast<uint8_t*>(
      dcnv2::align_up(reinterpret_cast<uintptr_t>(workspace), 256));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // events: entry, and per slot: inputs landed, forward done, output landed
  cudaEvent_t ev[1 + 3 * kHostSlots] = {};
  for (auto& e : ev)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      for (auto& f : ev) if (f) cudaEventDestroy(f);
      cudaGetLastError();
      return DCNV2_ERR_CUDA;
    }
  cudaEvent_t ev_entry = ev[0], *ev_in = ev + 1, *ev_fwd = ev_in + kHostSlots,
              *ev_out = ev_fwd + kHostSlots;
  const int N = desc->n;
  const uint8_t* xh = static_cast<const uint8_t*>(x_host);
  const uint8_t* oh = static_cast<const uint8_t*>(offset_host);
  const uint8_t* mh = static_cast<const uint8_t*>(mask_host);
  uint8_t* yh = static_cast<uint8_t*>(y_host);
  bool ok = cudaEventRecord(ev_entry, st) == cudaSuccess &&  // earlier work on `stream` first
            cudaStreamWaitEvent(cs->h2d, ev_entry, 0) == cudaSuccess &&
            cudaStreamWaitEvent(cs->d2h, ev_entry, 0) == cudaSuccess;
  // Chunk sizes: the first and the last chunk hold a quarter of the others' images (when the
  // batch spans more than two chunks). The upload before the first forward and the download
  // after the last one overlap nothing, so they are kept short; in between, uploads and
  // downloads share the bus in both directions.
  const int edge = hc.chunk >= 4 && N > 2 * hc.chunk ? hc.chunk / 4 : hc.chunk;
  auto chunk_at = [&](int n0) {
    const int left = N - n0;
    if (n0 == 0 || left <= edge) return left < edge ? left : edge;
    if (left - hc.chunk < edge) return left - edge;  // leaves `edge` images for the last chunk
    return hc.chunk;
  };
  int i = 0;
  for (int n0 = 0, nb = 0; ok && n0 < N; n0 += nb, ++i) {
    nb = chunk_at(n0);
    const int b = i % kHostSlots;
    uint8_t* slot = ws + b * hc.slot_bytes;
    // upload (slot b is free once the forward of chunk i - kHostSlots has read it)
    if (i >= kHostSlots) ok = ok && cudaStreamWaitEvent(cs->h2d, ev_fwd[b], 0) == cudaSuccess;
    ok = ok &&
         cudaMemcpyAsync(slot + hc.x_off, xh + n0 * hc.x_img, nb * hc.x_img,
                         cudaMemcpyHostToDevice, cs->h2d) == cudaSuccess &&
         cudaMemcpyAsync(slot + hc.off_off, oh + n0 * hc.off_img, nb * hc.off_img,
                         cudaMemcpyHostToDevice, cs->h2d) == cudaSuccess &&
         cudaMemcpyAsync(slot + hc.mask_off, mh + n0 * hc.mask_img, nb * hc.mask_img,
                         cudaMemcpyHostToDevice, cs->h2d) == cudaSuccess &&
         cudaEventRecord(ev_in[b], cs->h2d) == cudaSuccess;
    // forward (its y slot is free once the download of chunk i - kHostSlots has read it)
    ok = ok && cudaStreamWaitEvent(st, ev_in[b], 0) == cudaSuccess;
    if (i >= kHostSlots) ok = ok && cudaStreamWaitEvent(st, ev_out[b], 0) == cudaSuccess;
    if (ok) {
      dcnv2_desc d = *desc;
      d.n = nb;
      s = dcnv2_forward(&d, slot + hc.x_off, slot + hc.off_off, slot + hc.mask_off, weight, bias,
                        slot + hc.y_off, ws + hc.fwd_off, hc.fwd_bytes, x_scale, w_scale, stream);
      ok = s == DCNV2_OK && cudaEventRecord(ev_fwd[b], st) == cudaSuccess;
    }
    // download
    ok = ok && cudaStreamWaitEvent(cs->d2h, ev_fwd[b], 0) == cudaSuccess &&
         cudaMemcpyAsync(yh + n0 * hc.y_img, slot + hc.y_off, nb * hc.y_img,
                         cudaMemcpyDeviceToHost, cs->d2h) == cudaSuccess &&
         cudaEventRecord(ev_out[b], cs->d2h) == cudaSuccess;
  }
  // `stream` completes after every download
  for (int b = 0; ok && b < kHostSlots && b < i; ++b)
    ok = cudaStreamWaitEvent(st, ev_out[b], 0) == cudaSuccess;
  for (auto& e : ev) cudaEventDestroy(e);  // released once the work that uses them completes
  if (!ok) {
    cudaGetLastError();
    return s != DCNV2_OK ? s : DCNV2_ERR_CUDA;
  }
  return DCNV2_OK;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free forward. Some callers cannot call cudaMalloc while they run (a fixed memory
// plan, a latency-critical loop where an allocation would synchronise the device, a hard device
// memory budget), so they cannot provide the workspace dcnv2_forward needs. For them the scratch
// lives here, in one file-scope buffer that every GPU which loads this library holds until the
// process exits. Host code must not pass `dcnv2_static_scratch` itself to a kernel — in host code
// that name is only a stand-in for the device symbol — so its device address is looked up once
// per device with cudaGetSymbolAddress and cached. The forward that runs is dcnv2_forward,
// unchanged, with this buffer as its workspace; it rewrites every scratch byte it reads and its
// weight-pack launch (or the memset of the CUDA-core path) clears the error word, so nothing
// carries over from the previous call. Concurrent calls on one device race on the buffer.
static __device__ __align__(256) unsigned char dcnv2_static_scratch[DCNV2_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_scratch_mu;
void* g_static_scratch_addr[dcnv2::kMaxDevices] = {};

// Device address of the static buffer on the current device, looked up once per device with that
// device current (cudaGetSymbolAddress) and cached.
dcnv2_status static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return DCNV2_ERR_NO_DEVICE;
  }
  if (dev < 0 || dev >= dcnv2::kMaxDevices) return DCNV2_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_addr[dev]) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, dcnv2_static_scratch);
    if (e != cudaSuccess || !addr) {
      cudaGetLastError();
      return DCNV2_ERR_CUDA;
    }
    g_static_scratch_addr[dev] = addr;
  }
  *out = g_static_scratch_addr[dev];
  return DCNV2_OK;
}
}  // namespace

extern "C" dcnv2_status dcnv2_forward_static_scratch(const dcnv2_desc* desc, const void* x,
                                                     const void* offset, const void* mask,
                                                     const void* weight, const void* bias,
                                                     void* y, float x_scale, float w_scale,
                                                     dcnv2_stream_t stream) {
  Plan p;
  const dcnv2_status s = make_plan(desc, &p);
  if (s != DCNV2_OK) return s;
  if (p.ws_bytes > DCNV2_STATIC_SCRATCH_BYTES) return DCNV2_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const dcnv2_status a = static_scratch_address(&scratch);
  if (a != DCNV2_OK) return a;
  return dcnv2_forward(desc, x, offset, mask, weight, bias, y, scratch,
                       DCNV2_STATIC_SCRATCH_BYTES, x_scale, w_scale, stream);
}

// The error word of the static buffer lies at its start (the buffer is 256-byte aligned, which is
// where dcnv2_forward places the word of any workspace).
extern "C" dcnv2_status dcnv2_read_static_scratch_error(dcnv2_stream_t stream, int32_t* code) {
  if (!code) return DCNV2_ERR_INVALID_ARG;
  void* scratch = nullptr;
  const dcnv2_status a = static_scratch_address(&scratch);
  if (a != DCNV2_OK) return a;
  return dcnv2_read_device_error(scratch, stream, code);
}
