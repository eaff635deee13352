// conv_tc.cu -- FactorizedPrior transform layers as tcgen05 implicit GEMMs
// (sm_100a) and the C ABI of include/fcai_transforms.h.
//
// GEMM view of one layer: rows = output pixels (tiles of 128), columns =
// output channels (npad <= 256, one tile), K = taps x input channels.
//   * 5x5 stride-2 convolution: K runs over the 25 taps; for tap (ky, kx) and
//     a 64-channel block the A tile is one TMA load of an NHWC box whose
//     x/y element strides are 2, starting at (2*ox0 + kx - 2, 2*oy0 + ky - 2);
//     the zero padding is the TMA out-of-bounds fill.
//   * 5x5 stride-2 transposed convolution (padding 2, output padding 1): the
//     output splits into 4 phases (oy % 2, ox % 2); phase (py, px) is a
//     stride-1 convolution of the input with the taps ky = py (mod 2),
//     kx = px (mod 2), input offset ((py + 2 - ky) / 2, (px + 2 - kx) / 2).
//     Each phase is its own set of tiles, so no output pixel is written twice.
//   * the first analysis layer (3 input channels, fp32 NCHW image) builds
//     its A tile (K = 75 padded to 80) with four gather warps instead of TMA.
// The B tile (weights) is a TMA box of the packed [25][npad][cin] tensor.
//
// CTA organisation (persistent, one CTA per SM):
//   warps 0-3   epilogue: TMEM -> registers, bias, GDN/IGDN, store
//   warps 4-7   second epilogue group (first and scatter layers: the two
//               groups take alternate tiles)
//   warp 8      TMA producer
//   warp 9      MMA issuer; owns the TMEM allocation
//   warps 10-13 gather producers (first analysis layer only)
// The producer and MMA loops run on the whole warp, one elected lane issuing
// each instruction (first layer: on lane 0).  A shared-memory ring of as many
// stages as the free shared memory holds (mbarrier full/empty pairs) feeds
// the MMAs; two TMEM accumulator buffers let the epilogue of tile j overlap
// the main loop of tile j + 1.
//
// GDN fusion: the epilogue writes x^2 (bf16) of its 128 x 128 tile into
// shared memory in the MMA operand layout and issues a second GEMM
// x^2 @ gamma^T into TMEM; then y = x * rsqrt(beta + norm) (x * sqrt(...)
// for IGDN) is formed from the two accumulators and stored.
//
// Every mbarrier wait is bounded (1 s of %globaltimer); on a timeout the
// CTA records an error code, raises a shared abort flag so the other roles
// stop, drains its MMAs and frees its TMEM before returning.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "../../include/fcai_transforms.h"
#include "fcai_common.h"
#include "tc_ptx.h"

namespace ct {
using namespace tcx;

constexpr int kBM = 128;          // output pixels per tile (MMA M)
constexpr int kBK = 64;           // bf16 per K block: one 128-byte row
constexpr int kSmemBudget = 227 * 1024;  // dynamic shared memory per CTA
constexpr int kMaxStages = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kGatherThread0 = 320;  // warps 10-13
constexpr int kGatherThreads = 128;
// scatter layers: 8 x 16 input pixels per tile, of which the 6 x 14 core
// produces a 12 x 28 output block; cout = 3 (25 taps x 3 = 75 -> npad 80)
constexpr int kScatterTY = 8, kScatterTX = 16, kScatterCoreH = 6, kScatterCoreW = 14, kScatterCout = 3;
constexpr int kScatterMaxCinBlocks = 3;  // scatter layers keep their weights resident: cin <= 192
constexpr int kGatherK = 80;         // 3 x 5 x 5 = 75, padded to 5 MMAs of K = 16
// First layer, patch path: the tile's fp32 input window (3 channels x
// (2 TY + 3) rows x (2 TX + 8) columns, TX <= 64) arrives by one TMA load
// into one of two patch buffers.
constexpr int kPatchBuf = 11520;     // >= (2 TX + 8) * (2 TY + 3) * 3 * 4 for TX in {8, 16, 32, 64}, 128-aligned
constexpr int kPatchMaxTX = 64;
constexpr uint64_t kWaitNs = 1000000000ull;

enum Epi : int { kEpiBf16 = 0, kEpiGdn = 1, kEpiIgdn = 2, kEpiF32 = 3, kEpiF32Clamp = 4, kEpiScatter = 5 };

enum Err : int { kErrProducer = 1, kErrMma = 2, kErrEpilogue = 4, kErrGather = 8 };

struct Taps {
    int n;
    int8_t dy[25], dx[25];
    uint8_t w[25];
};

// Division by a per-launch constant d >= 1 as a multiply and shift, exact for
// 0 <= n < 2^31 (Granlund and Montgomery, "Division by invariant integers
// using multiplication", 1994, with N = 31): l = ceil(log2 d),
// m = floor(2^(31 + l) / d) + 1 < 2^32, n / d = (n * m) >> (31 + l).
struct FastDiv {
    uint32_t m, s;
};
static inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    return FastDiv{(uint32_t)((1ull << (31 + l)) / d + 1), 31 + l};
}
__device__ __forceinline__ int fdiv(int n, FastDiv f) { return (int)(((uint64_t)(uint32_t)n * f.m) >> f.s); }

struct ConvParams {
    int B, phases, tiles_x, tiles_y, TY, TX, GH, GW;  // per-phase GEMM pixel grid
    int step_x, step_y;                               // tile origin step (TX/TY, or the scatter core)
    int clamp;                                        // scatter epilogue: clamp to [0, 1]
    int stride;                                       // input step per GEMM pixel (2 conv, 1 deconv)
    int phase_major;                                  // tile order: phase slowest (see tile_coords)
    FastDiv div_tx, div_ty, div_ph, div_b;            // tiles_x, tiles_y, phases, B
    int cin, cout, cin_blocks;
    int out_c0, cout_total;                           // fp32 NCHW output: first channel written, channels per image
    int Hout, Wout, out_step;                         // output tensor size, output step per GEMM pixel
    int Hin, Win;
    int tiles_total;
    uint32_t tmem_cols, buf_stride;
    Taps taps[4];
    const float *bias;
    const float *beta;
    const float *x_in;   // first layer: fp32 NCHW [B, 3, Hin, Win]
    const void *wgather; // first layer: packed weight image
    int patch_tma;       // first layer: 1 = input windows by TMA (tmA maps x_in), 0 = direct loads
    int patch_w, patch_h;  // patch box: columns (2 TX + 8), rows (2 TY + 3)
    uint32_t patch_bytes;
    uint32_t *amax_out;      // optional: running max of |output| (float bits), for an FP8 consumer
    const float *act_scale;  // FP8 layers: device scale of the e4m3 input (amax / 448)
    float w_scale;           // FP8 layers: scale of the e4m3 weights
    int tma_store;       // GDN layers: the output tile leaves through TMA stores (tmO); 1 = 4-D
                         // NHWC box, 2 = transposed conv phase box (5-D view of the output)
    void *out;
    int *err;
};

// kPair: CTA pairs (cluster of 2) share each MMA (cta_group::2, M = 256):
// each CTA holds its 128 pixel rows of A and half of the N rows of B (and of
// gamma), so a CTA's operand ring carries a quarter less per MMA and fits more
// stages.
// kFp8: e4m3 operands (kind::f8f6f4) with per-tensor scales; a 128-byte K
// block then holds 128 channels instead of 64, and the tiles are byte for
// byte the bf16 ones.
template <int kNpad, int kEpi, bool kGather, bool kPair = false, bool kFp8 = false>
struct Layout {
    static constexpr bool kNorm = kEpi == kEpiGdn || kEpi == kEpiIgdn;
    static constexpr int kKe = kFp8 ? 2 * kBK : kBK;  // operand elements per 128-byte K block
    static constexpr int kNB = kPair ? kNpad / 2 : kNpad;  // B / gamma rows this CTA holds
    // Dual tiles (GDN / IGDN layers fed by TMA): a tile is 256 output
    // pixels, one A box of 256 rows per K step, and each K step issues two
    // M = 128 MMAs that share the B tile, so each byte of weights loaded
    // feeds twice the MMA work.
    // GDN over 192 channels.  TMA-fed layers (kXReg): 8 epilogue warps, two
    // column halves of 96, each thread keeps its pixel's conv outputs in
    // registers and the GDN GEMM writes the norm over them, so a buffer is
    // 192 TMEM columns and two fit.  The first layer keeps x in TMEM beside
    // the norm (384 columns, one buffer) and one input window.
    static constexpr bool kWide = kNorm && kNpad > 128;
    static constexpr bool kXReg = kWide && !kGather;
    static constexpr bool kDual = kNorm && !kGather && !kPair && !kWide;
    static constexpr int kRows = kDual ? 2 * kBM : kBM;  // output pixels per tile
    static constexpr int kA = kGather ? kBM * kGatherK * 2 : kRows * kBK * 2;
    // the scatter layer's weights (npad x cin, at most 4 K blocks) stay
    // resident, loaded once; its ring stages carry the A tile only
    static constexpr bool kWRes = kEpi == kEpiScatter;
    static constexpr int kB = (kGather || kWRes) ? 0 : kNB * kBK * 2;
    static constexpr int kWResBytes = kWRes ? kScatterMaxCinBlocks * kNpad * kBK * 2 : 0;
    static constexpr int kStage = kA + kB;
    static constexpr int kW = kGather ? kNpad * kGatherK * 2 : 0;
    static constexpr int kG = kNorm ? kNB * kNpad * 2 : 0;
    // Ping-pong epilogue (the first layer and the scatter layer, whose
    // epilogues outweigh their short mainloops): two groups of 4 warps take alternate tiles, each with its own
    // accumulator buffer, x^2 / staging tile and GDN barrier, so one tile's
    // GDN GEMM and stores overlap the other's passes.
    static constexpr bool kPingPong = (kGather && kNorm && !kWide) || kEpi == kEpiScatter;
    static constexpr int kPatchBufs = kWide ? 1 : 2;  // first layer: input window buffers
    static constexpr int kX2One = kNorm ? kBM * kNpad * 2 : 0;
    static constexpr int kX2 = kPingPong ? 2 * kX2One : kX2One;
    // scatter buffer: per input pixel its 25 taps as 16-byte quads {3
    // outputs, 0}: 100 words, whose quarter (25) is odd, so that 8
    // consecutive pixels' quads (a warp's 16-byte stores and loads) hit every
    // bank group once
    static constexpr int kSRow = 25 * 4;
    static constexpr int kSOne = kEpi == kEpiScatter ? kBM * kSRow * 4 : 0;
    static constexpr int kS = kPingPong ? 2 * kSOne : kSOne;
    // operand ring: as many stages as the shared memory left over holds
    // (more bytes in flight hide more of the TMA round trip)
    // Constant operands (not the scatter layer): a 128 x 16 "ones" A tile
    // (K columns 0 and 1 = 1.0) and B tiles holding, per output channel, the
    // bias (and GDN beta) split into bf16 hi + lo parts in K columns 0 and 1.
    // One K = 16 MMA of ones x bias starts each accumulation, and ones x beta
    // starts each GDN norm, so the epilogue adds neither.
    // FP8 layers scale the accumulator in the epilogue, so their bias is
    // added there (after the scale) instead of folded.
    static constexpr bool kFoldBias = kEpi != kEpiScatter && !kFp8;
    static constexpr bool kFold = kFoldBias || kNorm;  // the ones tile exists
    static constexpr int kConstRow = 32;  // bytes per row of a K = 16 no-swizzle tile
    static constexpr int kOnes = kFold ? kBM * kConstRow : 0;
    static constexpr int kBiasB = kFoldBias ? kNB * kConstRow : 0;
    static constexpr int kBetaB = kNorm ? kNB * kConstRow : 0;
    static constexpr int kFixedBytes = kWResBytes + kOnes + kBiasB + kBetaB + kW + kG + kX2 +
                                       kS + (kGather ? kPatchBufs * kPatchBuf : 0) +
                                       2 * kNpad * 4 + (2 * kMaxStages + 11) * 8 + 32 + 1024;
    static constexpr int kStagesRaw = (kSmemBudget - kFixedBytes) / kStage;
    static constexpr int kStages = kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw;
    static constexpr int offWRes = kStages * kStage;
    static constexpr int offW = offWRes + kWResBytes;
    static constexpr int offG = offW + kW;
    static constexpr int offX2 = offG + kG;
    static constexpr int offS = offX2 + kX2;
    static constexpr int kP = kGather ? kPatchBufs * kPatchBuf : 0;
    static constexpr int offPatch = offS + kS;
    static constexpr int offOnes = offPatch + kP;
    static constexpr int offBiasB = offOnes + kOnes;
    static constexpr int offBetaB = offBiasB + kBiasB;
    static constexpr int offBias = offBetaB + kBetaB;
    static constexpr int offBeta = offBias + kNpad * 4;
    static constexpr int offBar = (offBeta + kNpad * 4 + 7) & ~7;
    // TMEM accumulator buffers: 2, or 4 for the scatter layer (128 columns
    // each), whose short tiles would otherwise make the MMA wait for the
    // epilogue of the tile before last
    static constexpr int kAccBufs = kEpi == kEpiScatter ? 4 : (kWide && !kXReg ? 1 : 2);
    static constexpr int kBars = 2 * kStages + 2 * kAccBufs + 4 + (kGather ? 4 : 0) + (kPair ? 1 : 0);
    static_assert(kStages >= 2, "operand ring");
    static constexpr int offSlot = offBar + kBars * 8;
    static constexpr int kBytes = offSlot + 32;
    static constexpr int kAlloc = kBytes + 1024;  // base alignment slack
    static constexpr int kThreads = kGather ? 448 : 320;
    // Epilogue warps: one per TMEM lane quarter where the mainloop bounds the
    // layer (fewer warps competing with the MMA warp for issue slots), two
    // (column halves) where the epilogue is the heavy part: the first layer
    // (K = 80) and the scatter layer.
    static constexpr int kEpiWarps = (kGather || kEpi == kEpiScatter || kDual || kXReg) ? 8 : 4;
    static constexpr int kEpiThreads = kEpiWarps * 32;
    // column split between the two epilogue warps of a lane quarter
    static constexpr int kSplit = kEpiWarps == 8 && !kPingPong && kNpad >= 32 ? (kNpad / 2) / 16 * 16 : kNpad;
    static constexpr int kGroups = kPingPong ? 2 : 1;
    // Producer and MMA loops run on the whole warp (warp-uniform operands,
    // one elected lane issues) where TMA feeds the operand ring; the first
    // layer, whose epilogue and gather warps bound it, keeps them on one lane
    // so that its loops take fewer issue slots from those warps.
    static constexpr bool kWarpIssue = !kGather;
    static constexpr int kGroupThreads = kEpiThreads / kGroups;
    static_assert(kEpi != kEpiScatter || kNpad == 25 * kScatterCout + 5, "scatter instance is built for cout = 3");
    static_assert(kA % 1024 == 0 || kGather, "A stage alignment");
    static_assert(offPatch % 128 == 0 && kPatchBuf % 128 == 0, "patch buffer alignment");
    static_assert(offOnes % 128 == 0 && kOnes % 128 == 0 && kBiasB % 128 == 0, "constant tile alignment");
    static_assert(kB % 1024 == 0, "B stage alignment");
    static_assert(kWResBytes % 1024 == 0 && (kNpad * kBK * 2) % 1024 == 0 || !kWRes, "resident weight alignment");
    static_assert(!kNorm || kNpad == 128 || kNpad == 192, "GDN fusion is built for 128 or 192 channels");
    static_assert(!kWide || !kPair, "192-channel GDN has no CTA-pair instance");
    static_assert(!kFp8 || (!kGather && !kPair && kEpi != kEpiScatter), "FP8 instances: TMA-fed single-CTA layers");
    static_assert(!kPair || (!kGather && kEpi != kEpiScatter && kNB % 8 == 0), "pair instances: TMA operands");
    static_assert(kNpad % 16 == 0 && kNpad >= 16 && kNpad <= 256, "MMA N");
};

// Tile order: x fastest, then y, then phase, then image (an image's phases
// close together in time, so its input stays in L2); or, with phase_major
// (transposed IGDN layers only; other instances compile without the
// branch), image before phase: the CTAs' round-robin shares then hold about
// one tile of each phase (9, 6, 6 and 4 taps) instead of runs of one phase,
// which balances layers of few tiles per CTA.
template <bool kPhaseMajor>
__device__ __forceinline__ void tile_coords(const ConvParams &p, int tile, int &b, int &ph, int &gy0, int &gx0) {
    int rest = fdiv(tile, p.div_tx);
    const int tx = tile - rest * p.tiles_x;
    int r2 = fdiv(rest, p.div_ty);
    const int ty = rest - r2 * p.tiles_y;
    rest = r2;
    if (kPhaseMajor && p.phase_major) {
        ph = fdiv(rest, p.div_b);
        b = rest - ph * p.B;
    } else {
        b = fdiv(rest, p.div_ph);
        ph = rest - b * p.phases;
    }
    gy0 = ty * p.step_y;
    gx0 = tx * p.step_x;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

// |x| of bf16 values orders like its bits without the sign, so the running
// max of a thread's outputs is kept as two 16-bit lanes (vmaxu2) and folded
// into one float at the end.
__device__ __forceinline__ uint32_t amax_bf16x2(uint32_t am2, uint32_t packed) {
    return __vmaxu2(am2, packed & 0x7FFF7FFFu);
}
// The warp's max |output| into *dst (float bits; all 32 lanes call it).
__device__ __forceinline__ void amax_flush(uint32_t *dst, uint32_t am2) {
    uint32_t am = max(am2 & 0xFFFFu, am2 >> 16) << 16;
    am = __reduce_max_sync(0xffffffffu, am);
    if (dst && (threadIdx.x & 31) == 0) atomicMax(dst, am);
}

__device__ __forceinline__ float4 ld_shared_v4f(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// One lane (W = false) or the whole warp (W = true) runs the calling loop.
template <bool W>
__device__ __forceinline__ bool wait_for(uint64_t *bar, uint32_t parity, volatile int *abort, bool cluster = false) {
    return W ? mbar_wait_warp(bar, parity, abort, kWaitNs, cluster) : mbar_wait(bar, parity, abort, kWaitNs, cluster);
}
template <bool W>
__device__ __forceinline__ bool aborted(volatile int *abort) {
    return W ? __any_sync(0xffffffffu, *abort != 0) : *abort != 0;
}
template <bool W>
__device__ __forceinline__ void mma_issue(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (W) mma_bf16_w(d, a, b, idesc, acc);
    else mma_bf16(d, a, b, idesc, acc);
}
template <bool W>
__device__ __forceinline__ void mma_issue_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (W) mma_bf16_pair_w(d, a, b, idesc, acc);
    else mma_bf16_pair(d, a, b, idesc, acc);
}
template <bool W>
__device__ __forceinline__ void mma_issue_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (W) mma_e4m3_w(d, a, b, idesc, acc);
    else mma_e4m3(d, a, b, idesc, acc);
}
template <bool W>
__device__ __forceinline__ void commit_to(uint64_t *bar) {
    if (W) mma_commit_w(bar);
    else mma_commit(bar);
}
template <bool W>
__device__ __forceinline__ void commit_pair_to(uint64_t *bar) {
    if (W) mma_commit_pair_both_w(bar, 3);
    else mma_commit_pair_both(bar, 3);
}

__device__ __forceinline__ void fail(const ConvParams &p, volatile int *abort, int code) {
    *abort = 1;
    if (p.err) atomicOr(p.err, code);
}

template <int kNpad, int kEpi, bool kGather, bool kPair, bool kFp8>
__global__ void __launch_bounds__(Layout<kNpad, kEpi, kGather, kPair, kFp8>::kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmO,
                   const ConvParams p) {
    using Lay = Layout<kNpad, kEpi, kGather, kPair, kFp8>;
    constexpr bool kNorm = Lay::kNorm;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Lay::offBar);
    uint64_t *full = bars;
    constexpr int kStages = Lay::kStages;
    uint64_t *empty = bars + kStages;
    uint64_t *accf = bars + 2 * kStages;
    uint64_t *acce = accf + Lay::kAccBufs;
    uint64_t *g2bar = acce + Lay::kAccBufs;   // GDN GEMM done (one per epilogue group)
    uint64_t *cbar = g2bar + 2;
    uint64_t *dbar = cbar + 1;  // abort path: drains this CTA's MMAs
    uint64_t *pfull = dbar + 1;   // first layer: patch buffer loaded (2)
    uint64_t *pempty = pfull + 2; // first layer: patch buffer read by all gather threads (2)
    uint64_t *x2full = dbar + 1;  // pairs (rank 0): both CTAs wrote their x^2 tile
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Lay::offSlot);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + Lay::offSlot + 4);
    volatile int *epi_ok = reinterpret_cast<volatile int *>(smem + Lay::offSlot + 8);
    float *s_bias = reinterpret_cast<float *>(smem + Lay::offBias);
    float *s_beta = reinterpret_cast<float *>(smem + Lay::offBeta);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Pairs: CTA `rank` of the cluster takes pixel sub-tile `rank` of each
    // pair tile; rank 0 (the leader) issues all MMAs of the pair.
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int unit0 = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // first tile (pair tile) of this CTA
    const int unit_step = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int sub_x = kPair ? (int)rank * p.TX : 0;                      // sub-tile origin within a pair tile

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kGather ? kGatherThreads : 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < Lay::kAccBufs; ++b) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], kPair ? 2 : Lay::kGroupThreads);  // pairs: one arrival per CTA's epilogue
        }
        if (kPair) mbar_init(x2full, 2);
        mbar_init(&g2bar[0], 1);
        mbar_init(&g2bar[1], 1);
        mbar_init(cbar, 1);
        // the MMA thread and each epilogue thread that issues GDN GEMMs
        mbar_init(dbar, 1 + ((Lay::kPingPong || Lay::kDual) ? 2 : 1));
        if (kGather) {
            for (int b = 0; b < 2; ++b) {
                mbar_init(&pfull[b], 1);
                mbar_init(&pempty[b], kGatherThreads);
            }
        }
        *abort = 0;
        fence_barrier_init();
    }
    for (int i = threadIdx.x; i < kNpad; i += blockDim.x) {
        s_bias[i] = i < p.cout ? p.bias[i] : 0.f;
        if (kNorm) s_beta[i] = i < p.cout ? p.beta[i] : 1.f;
    }
    if (Lay::kFold) {
        // no-swizzle K-major tiles: row r's K columns 0-7 at
        // (r / 8) * 256 + (r % 8) * 16, columns 8-15 128 bytes further
        for (int r = threadIdx.x; r < kBM + 2 * Lay::kNB; r += blockDim.x) {
            uint32_t w0;
            unsigned char *tile;
            int row;
            if (r < kBM) {
                w0 = pack_bf16x2(1.f, 1.f);
                tile = smem + Lay::offOnes;
                row = r;
            } else {
                row = (r - kBM) % Lay::kNB;
                const bool is_beta = r >= kBM + Lay::kNB;
                if (is_beta && !kNorm) continue;
                if (!is_beta && !Lay::kFoldBias) continue;
                const int c = (int)rank * Lay::kNB + row;  // pairs: this CTA's half of the channels
                const float v = is_beta ? (c < p.cout ? p.beta[c] : 1.f) : (c < p.cout ? p.bias[c] : 0.f);
                const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
                w0 = (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
                tile = smem + (is_beta ? Lay::offBetaB : Lay::offBiasB);
            }
            uint4 *q = reinterpret_cast<uint4 *>(tile + (row >> 3) * 256 + (row & 7) * 16);
            q[0] = make_uint4(w0, 0u, 0u, 0u);
            q[8] = make_uint4(0u, 0u, 0u, 0u);  // K columns 8-15, 128 bytes on
        }
        fence_proxy_async_smem();  // the tensor core reads these tiles
    }
    if (warp == kMmaWarp) {
        if (kPair) {
            tmem_alloc_pair(tmem_slot, p.tmem_cols);  // same warp and slot in both CTAs
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, p.tmem_cols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // pairs: both CTAs' barriers exist before any remote arrive or load names them
    if (kPair) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        // one-time operands from lane 0; the operand ring from the whole warp
        // (one elected lane issues each load); the first layer's input
        // windows from lane 0
        const uint32_t cbytes = (kNorm ? Lay::kG : 0) + (kGather ? Lay::kW : 0) +
                                (Lay::kWRes ? (uint32_t)(p.cin_blocks * kNpad * kBK * 2) : 0u);
        if (lane == 0) {
            if (!kGather) {
                tma_prefetch_desc(&tmA);
                tma_prefetch_desc(&tmW);
            } else if (p.patch_tma) {
                tma_prefetch_desc(&tmA);
            }
            if (cbytes) {
                mbar_arrive_expect_tx(cbar, cbytes);
                if (kNorm) {  // pairs: this CTA's half of the gamma rows
                    for (int kb = 0; kb < kNpad / kBK; ++kb)
                        tma_load_3d(smem + Lay::offG + kb * (Lay::kNB * 128), &tmG, cbar, kb * kBK,
                                    (int)rank * Lay::kNB, 0);
                }
                if (kGather) bulk_load(smem + Lay::offW, p.wgather, Lay::kW, cbar);
                if (Lay::kWRes)
                    for (int cb = 0; cb < p.cin_blocks; ++cb)
                        tma_load_3d(smem + Lay::offWRes + cb * (kNpad * kBK * 2), &tmW, cbar, cb * kBK, 0, 0);
            }
        }
        __syncwarp();
        if (!kGather) {
            static_assert(kGather || Lay::kWarpIssue, "the operand ring is fed warp-wide");
            uint32_t it = 0;
            int last_round[kStages];
            for (int s = 0; s < kStages; ++s) last_round[s] = -1;
            bool stop = false;
            for (int tile = unit0; tile < p.tiles_total && !stop; tile += unit_step) {
                int b, ph, gy0, gx0;
                tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
                gx0 += sub_x;
                const Taps &tp = p.taps[ph];
                for (int t = 0; t < tp.n && !stop; ++t) {
                    const int ix = gx0 * p.stride + tp.dx[t];
                    const int iy = gy0 * p.stride + tp.dy[t];
                    for (int cb = 0; cb < p.cin_blocks; ++cb, ++it) {
                        const int s = it % kStages;
                        const uint32_t r = it / kStages;
                        if (!wait_for<true>(&empty[s], (r & 1) ^ 1, abort)) {
                            if (lane == 0) fail(p, abort, kErrProducer);
                            stop = true;
                            break;
                        }
                        unsigned char *st = smem + s * Lay::kStage;
                        if (kPair) {
                            if (lane == 0) {
                                // both CTAs' bytes count on the leader's full[s]
                                const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                                if (leader) mbar_arrive_expect_tx(&full[s], 2 * Lay::kStage);
                                tma_load_4d_pair(st, &tmA, fb, cb * kBK, ix, iy, b);
                                tma_load_3d_pair(st + Lay::kA, &tmW, fb, cb * kBK, (int)rank * Lay::kNB, tp.w[t]);
                            }
                            __syncwarp();
                        } else {
                            mbar_arrive_expect_tx_w(&full[s], Lay::kStage);
                            tma_load_4d_w(st, &tmA, &full[s], cb * Lay::kKe, ix, iy, b);
                            if (!Lay::kWRes) tma_load_3d_w(st + Lay::kA, &tmW, &full[s], cb * Lay::kKe, 0, tp.w[t]);
                        }
                        last_round[s] = (int)r;
                    }
                }
                if (aborted<true>(abort)) stop = true;
            }
            if (lane == 0 && *abort && leader) {
                // let the loads in flight land before the CTA exits (pairs:
                // the leader's full[s] also counts the peer's loads)
                for (int s = 0; s < kStages; ++s)
                    if (last_round[s] >= 0) mbar_wait(&full[s], (uint32_t)last_round[s] & 1, nullptr, kWaitNs / 10);
            }
        }
        if (kGather && p.patch_tma && lane == 0) {
            // input windows: patch buffer it % kPatchBufs for the CTA's it-th tile
            uint32_t it = 0;
            int last_round[2] = {-1, -1};
            for (int tile = blockIdx.x; tile < p.tiles_total && !*abort; tile += gridDim.x, ++it) {
                int b, ph, gy0, gx0;
                tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
                const int pb = (int)(it % Lay::kPatchBufs);
                const uint32_t r = it / Lay::kPatchBufs;
                if (!mbar_wait(&pempty[pb], (r & 1) ^ 1, abort, kWaitNs)) {
                    fail(p, abort, kErrProducer);
                    break;
                }
                mbar_arrive_expect_tx(&pfull[pb], p.patch_bytes);
                // x starts 4 columns left of the window's first input column
                // (2 gx0 - 2): a multiple of 4 floats, as TMA requires; the
                // rows above / columns left of the image read as zeros
                tma_load_4d(smem + Lay::offPatch + pb * kPatchBuf, &tmA, &pfull[pb], 2 * gx0 - 4, 2 * gy0 - 2, 0,
                            b);
                last_round[pb] = (int)r;
            }
            if (*abort) {
                for (int pb = 0; pb < 2; ++pb)
                    if (last_round[pb] >= 0)
                        mbar_wait(&pfull[pb], (uint32_t)last_round[pb] & 1, nullptr, kWaitNs / 10);
            }
        }
        if (lane == 0 && cbytes && *abort) mbar_wait(cbar, 0, nullptr, kWaitNs / 10);
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        // Lane 0, or the whole warp with one elected lane issuing (kWarpIssue);
        // pairs: the leader CTA alone, whose commits arrive in both CTAs.
        constexpr bool W = Lay::kWarpIssue;
        if (leader && (W || lane == 0)) {
            const uint32_t idesc = idesc_bf16(kPair ? 2 * kBM : kBM, kNpad);
            const uint32_t idesc_main = kFp8 ? idesc_e4m3(kBM, kNpad) : idesc;
            bool consts = !(kGather || Lay::kWRes);  // the first layer's / scatter layer's weights arrive once
            uint32_t it = 0;
            int j = 0;
            for (int tile = unit0; tile < p.tiles_total && !aborted<W>(abort); tile += unit_step, ++j) {
                if (!consts) {
                    if (!wait_for<W>(cbar, 0, abort)) {
                        if (lane == 0) fail(p, abort, kErrMma);
                        break;
                    }
                    consts = true;
                }
                int b, ph, gy0, gx0;
                tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
                const int buf = j % Lay::kAccBufs;
                const uint32_t use = j / Lay::kAccBufs;
                if (!wait_for<W>(&acce[buf], (use & 1) ^ 1, abort, kPair)) {
                    if (lane == 0) fail(p, abort, kErrMma);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + buf * p.buf_stride;
                const int ksteps = kGather ? 1 : p.taps[ph].n * p.cin_blocks;
                bool ok = true;
                for (int ks = 0; ks < ksteps; ++ks, ++it) {
                    const int s = it % kStages;
                    const uint32_t r = it / kStages;
                    if (!wait_for<W>(&full[s], r & 1, abort)) {
                        if (lane == 0) fail(p, abort, kErrMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + s * Lay::kStage);
                    // the tile's accumulator starts as the bias (ones x bias)
                    const bool first = ks == 0;
                    if (Lay::kFoldBias && first) {
                        const uint64_t od = smem_desc(smem_u32(smem + Lay::offOnes), 128, 256, 0);
                        const uint64_t bd = smem_desc(smem_u32(smem + Lay::offBiasB), 128, 256, 0);
                        if (kPair) mma_issue_pair<W>(d, od, bd, idesc, 0);
                        else mma_issue<W>(d, od, bd, idesc, 0);
                        if (Lay::kDual) mma_issue<W>(d + kBM, od, bd, idesc, 0);  // second half's columns
                    }
                    const bool fresh = first && !Lay::kFoldBias;  // the first MMA overwrites the accumulator
                    if (kGather) {
                        const uint32_t w0 = smem_u32(smem + Lay::offW);
#pragma unroll
                        for (int kk = 0; kk < kGatherK / 16; ++kk)
                            mma_issue<W>(d, smem_desc(a0 + kk * 256, 128, 1280, 0),
                                         smem_desc(w0 + kk * 256, 128, 1280, 0), idesc, !(fresh && kk == 0));
                    } else if (kPair) {
                        const uint32_t b0 = a0 + Lay::kA;
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk)
                            mma_issue_pair<W>(d, smem_desc(a0 + kk * 32, 16, 1024, 2),
                                              smem_desc(b0 + kk * 32, 16, 1024, 2), idesc, !(fresh && kk == 0));
                    } else {
                        // resident weights: K block ks (the scatter layer has one tap)
                        const uint32_t b0 = Lay::kWRes ? smem_u32(smem + Lay::offWRes) + ks * (kNpad * kBK * 2)
                                                       : a0 + Lay::kA;
                        if constexpr (Lay::kWRes) {
                            // the scatter layer's short N = 80 MMAs: the K
                            // block's four in one issue block (one elect, the
                            // descriptors advanced inside it), which issues
                            // them faster than four calls; the dual-tile
                            // layers ran slower that way and keep the loop
                            mma_kblock<W, kFp8>(d, smem_desc(a0, 16, 1024, 2), smem_desc(b0, 16, 1024, 2), idesc_main,
                                                !fresh);
                        } else {
#pragma unroll
                            // 4 MMAs per 128-byte K block: K = 16 bf16 or 32 e4m3 each
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint64_t bd = smem_desc(b0 + kk * 32, 16, 1024, 2);
                                const uint64_t ad = smem_desc(a0 + kk * 32, 16, 1024, 2);
                                const uint32_t acc = !(fresh && kk == 0);
                                if (kFp8) mma_issue_f8<W>(d, ad, bd, idesc_main, acc);
                                else mma_issue<W>(d, ad, bd, idesc, acc);
                                // dual tiles: rows 128-255 of A into the second half's columns
                                if (Lay::kDual) {
                                    const uint64_t ad1 = smem_desc(a0 + kBM * 128 + kk * 32, 16, 1024, 2);
                                    if (kFp8) mma_issue_f8<W>(d + kBM, ad1, bd, idesc_main, acc);
                                    else mma_issue<W>(d + kBM, ad1, bd, idesc, acc);
                                }
                            }
                        }
                    }
                    // frees the stage (pairs: in both CTAs) once these MMAs have read it
                    if (kPair) commit_pair_to<W>(&empty[s]);
                    else commit_to<W>(&empty[s]);
                }
                if (!ok) break;
                if (kPair) commit_pair_to<W>(&accf[buf]);
                else commit_to<W>(&accf[buf]);
            }
            if (W) __syncwarp();
        }
    } else if (warp < Lay::kEpiWarps) {
        // ------------------------------------------------------------ epilogue
        if constexpr (Lay::kDual && kEpi == kEpiIgdn) {
            // Two epilogue variants of dual tiles, chosen by measurement (the
            // same build, batch 24, alternating runs): the IGDN layers (short
            // phase mainloops of 4-9 taps) run faster when the two groups do
            // not take turns with one operand tile (g_s.4 0.477 -> 0.461 ms,
            // g_s.2 0.130 -> 0.125 ms); the GDN layers (25-tap mainloops that
            // already hide the epilogue) run faster with one shared tile and
            // a single GDN GEMM per half (g_a.2 0.388 against 0.396 ms).
            //
            // Dual tiles: rows 0-127 of the tile (TMEM columns [0, 128) of the
            // buffer) belong to group 0 (warps 0-3), rows 128-255 (columns
            // [128, 256)) to group 1 (warps 4-7).  Each thread keeps its
            // pixel's 128 conv outputs in registers, so the GDN GEMM writes
            // the norm over them in TMEM.  Each group owns one 16 KB half of
            // the x^2 / staging area: the GDN GEMM runs in two K halves (x^2
            // of channels 0-63, then of 64-127, through the group's half), and
            // the output leaves in two 64-channel boxes staged there in turn,
            // so the two groups never wait for each other inside a tile.
            // Named barriers: 1 + h (group h), 3 (all 256 threads, tile
            // start).  Every barrier of a tile is taken by every thread of its
            // group, whatever the outcome of the waits (the work between them
            // is what the outcome skips).
            const int h = warp >> 2;
            const int m = threadIdx.x & 127;
            const bool hleader = m == 0;
            const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
            const uint32_t x2 = smem_u32(smem + Lay::offX2) + (uint32_t)h * (kBM * 128);  // this group's half
            volatile int *t_ok = epi_ok;
            volatile int *h_ok = epi_ok + 1 + h;
            uint32_t am2 = 0;  // max |output| of this thread's valid pixels (amax_out)
            bool consts = false;
            int j = 0;
            for (int tile = unit0; tile < p.tiles_total; tile += unit_step, ++j) {
                int b, ph, gy0, gx0;
                tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
                const int buf = j & 1;
                const uint32_t use = j >> 1;
                if (threadIdx.x == 0) {
                    bool ok = !*abort;
                    if (ok && !consts) ok = mbar_wait(cbar, 0, abort, kWaitNs);
                    if (ok) ok = mbar_wait(&accf[buf], use & 1, abort, kWaitNs);
                    if (!ok) fail(p, abort, kErrEpilogue);
                    *t_ok = ok ? 1 : 0;
                }
                // the group has passed its last read of h_ok for the previous
                // tile (its last barrier), so the leader may reset it here
                if (hleader) *h_ok = 1;
                // each group's leader saw its previous tile's stores read its
                // half before it got here
                named_barrier_sync(3, 2 * kBM);
                if (!*t_ok) break;
                consts = true;
                tc_fence_after();
                const uint32_t dcol = tmem_base + buf * p.buf_stride + h * kBM;  // this half's columns
                uint32_t xv[kNpad / 16][16];
#pragma unroll
                for (int k = 0; k < kNpad / 16; ++k) tmem_ld16(dcol + lane_addr + k * 16, xv[k]);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < kNpad / 16; ++k) tmem_regs_ready(xv[k]);
                if (kFp8) {
                    // x = (s_x s_w) * accumulator + bias
                    const float sc = *p.act_scale * p.w_scale;
#pragma unroll
                    for (int k = 0; k < kNpad / 16; ++k)
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            xv[k][e] = __float_as_uint(fmaf(__uint_as_float(xv[k][e]), sc, s_bias[k * 16 + e]));
                }
                // norm = beta (ones x beta) + x^2 gamma^T in two K halves of
                // 64 channels through this group's 16 KB operand tile
#pragma unroll
                for (int q = 0; q < kNpad / kBK; ++q) {
                    if (*h_ok) {
#pragma unroll
                        for (int k = q * (kBK / 16); k < (q + 1) * (kBK / 16); ++k) {
#pragma unroll
                            for (int hh = 0; hh < 2; ++hh) {
                                uint32_t w[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float a = __uint_as_float(xv[k][hh * 8 + 2 * e]);
                                    const float c = __uint_as_float(xv[k][hh * 8 + 2 * e + 1]);
                                    w[e] = pack_bf16x2(a * a, c * c);
                                }
                                const int chunk = ((k * 16 + hh * 8) % kBK) / 8;
                                st_shared_v4(x2 + m * 128 + ((chunk ^ (m & 7)) << 4), w[0], w[1], w[2], w[3]);
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    tc_fence_before();  // the TMEM loads above precede the GEMM that overwrites those columns
                    named_barrier_sync(1 + h, kBM);
                    if (hleader && *h_ok) {
                        tc_fence_after();
                        const uint32_t g0 = smem_u32(smem + Lay::offG) + q * (kNpad * 128);
                        const uint32_t idesc = idesc_bf16(kBM, kNpad);
                        if (q == 0)
                            mma_bf16(dcol, smem_desc(smem_u32(smem + Lay::offOnes), 128, 256, 0),
                                     smem_desc(smem_u32(smem + Lay::offBetaB), 128, 256, 0), idesc, 0);
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk)
                            mma_bf16(dcol, smem_desc(x2 + kk * 32, 16, 1024, 2), smem_desc(g0 + kk * 32, 16, 1024, 2),
                                     idesc, 1);
                        mma_commit(&g2bar[h]);
                        // two GEMM halves a tile: the q-th completion of the tile has parity q
                        const bool ok = mbar_wait(&g2bar[h], (uint32_t)q & 1u, abort, kWaitNs);
                        if (!ok) fail(p, abort, kErrEpilogue);
                        *h_ok = ok ? 1 : 0;
                    }
                    named_barrier_sync(1 + h, kBM);
                }
                const bool hok = *h_ok != 0;
                tc_fence_after();
                // y = x * rsqrt(norm) (IGDN: x * sqrt(norm)), one 64-channel box at
                // a time: staged in this group's half and stored by TMA, or
                // stored straight to global memory
                const int row = h * kBM + m;
                const int ty = row / p.TX, tx = row - ty * p.TX;
                const int gy = gy0 + ty, gx = gx0 + tx;
                const bool valid = gy < p.GH && gx < p.GW;
                const int oy = gy * p.out_step + (p.phases == 4 ? (ph >> 1) : 0);
                const int ox = gx * p.out_step + (p.phases == 4 ? (ph & 1) : 0);
                __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                      (((int64_t)b * p.Hout + oy) * p.Wout + ox) * kNpad;
                const int hy = gy0 + h * (p.TY / 2);  // this half: TY / 2 rows of the tile
#pragma unroll
                for (int kb = 0; kb < kNpad / kBK; ++kb) {
                    if (hok) {
                        uint32_t nv[2][16];
                        constexpr int kPer = kBK / 16;
                        tmem_ld16(dcol + lane_addr + kb * kBK, nv[0]);
#pragma unroll
                        for (int i = 0; i < kPer; ++i) {
                            const int k = kb * kPer + i;
                            tmem_wait_ld();
                            tmem_regs_ready(nv[i & 1]);
                            if (i + 1 < kPer) tmem_ld16(dcol + lane_addr + (k + 1) * 16, nv[(i + 1) & 1]);
                            uint32_t o[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float n0 = __uint_as_float(nv[i & 1][2 * e]);
                                const float n1 = __uint_as_float(nv[i & 1][2 * e + 1]);
                                const float r0 = kEpi == kEpiIgdn ? sqrt_approx(n0) : rsqrt_approx(n0);
                                const float r1 = kEpi == kEpiIgdn ? sqrt_approx(n1) : rsqrt_approx(n1);
                                o[e] = pack_bf16x2(__uint_as_float(xv[k][2 * e]) * r0,
                                                   __uint_as_float(xv[k][2 * e + 1]) * r1);
                                if (valid) am2 = amax_bf16x2(am2, o[e]);
                            }
                            if (p.tma_store) {
#pragma unroll
                                for (int hh = 0; hh < 2; ++hh) {
                                    const int chunk = ((k * 16 + hh * 8) % kBK) / 8;
                                    st_shared_v4(x2 + m * 128 + ((chunk ^ (m & 7)) << 4), o[hh * 4], o[hh * 4 + 1],
                                                 o[hh * 4 + 2], o[hh * 4 + 3]);
                                }
                            } else if (valid) {
                                uint4 *dst = reinterpret_cast<uint4 *>(orow + k * 16);
                                dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                                dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                            }
                        }
                    }
                    if (kb == kNpad / kBK - 1) {
                        tc_fence_before();
                        mbar_arrive(&acce[buf]);  // this thread is done with the accumulator
                    }
                    fence_proxy_async_smem();
                    named_barrier_sync(1 + h, kBM);
                    if (hleader && p.tma_store) {
                        if (hok) {
                            const uint8_t *stg = smem + Lay::offX2 + h * (kBM * 128);
                            if (p.tma_store == 2)
                                tma_store_5d(&tmO, stg, kb * kBK, ph & 1, gx0, ph >> 1, b * p.GH + hy);
                            else
                                tma_store_4d(&tmO, stg, kb * kBK, gx0, hy, b);
                            bulk_commit_group();
                        }
                        bulk_wait_read_all();  // the half may be rewritten (next box or next tile's x^2)
                    }
                    if (kb + 1 < kNpad / kBK) named_barrier_sync(1 + h, kBM);
                }
            }
            if (hleader && p.tma_store) bulk_wait_all();  // stores complete before the CTA exits
            if (p.amax_out) amax_flush(p.amax_out, am2);
        } else if constexpr (Lay::kDual) {
            // Dual tiles: rows 0-127 of the tile (TMEM columns [0, 128) of the
            // buffer) belong to group 0 (warps 0-3), rows 128-255 (columns
            // [128, 256)) to group 1 (warps 4-7).  Each thread keeps its
            // pixel's 128 conv outputs in registers, so the GDN GEMM writes
            // the norm over them in TMEM.  The groups use the one x^2 /
            // staging tile in turn, group 0 first.  Named barriers: 1 + h
            // (group h), 3 (all 256 threads, tile start), 4 (group 0 hands the
            // tile to group 1).  No thread leaves the loop between the tile
            // start and its end, so every barrier always meets all its threads.
            const int h = warp >> 2;
            const int m = threadIdx.x & 127;
            const bool hleader = m == 0;
            const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
            const uint32_t x2 = smem_u32(smem + Lay::offX2);
            volatile int *t_ok = epi_ok;
            volatile int *h_ok = epi_ok + 1 + h;
            uint32_t am2 = 0;  // max |output| of this thread's valid pixels (amax_out)
            bool consts = false;
            int j = 0;
            for (int tile = unit0; tile < p.tiles_total; tile += unit_step, ++j) {
                int b, ph, gy0, gx0;
                tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
                const int buf = j & 1;
                const uint32_t use = j >> 1;
                if (threadIdx.x == 0) {
                    bool ok = !*abort;
                    if (ok && !consts) ok = mbar_wait(cbar, 0, abort, kWaitNs);
                    if (ok) ok = mbar_wait(&accf[buf], use & 1, abort, kWaitNs);
                    if (!ok) fail(p, abort, kErrEpilogue);
                    *t_ok = ok ? 1 : 0;
                }
                // group 1's leader saw its stores read the x^2 tile before it got here
                named_barrier_sync(3, 2 * kBM);
                if (!*t_ok) break;
                consts = true;
                tc_fence_after();
                const uint32_t dcol = tmem_base + buf * p.buf_stride + h * kBM;  // this half's columns
                uint32_t xv[kNpad / 16][16];
#pragma unroll
                for (int k = 0; k < kNpad / 16; ++k) tmem_ld16(dcol + lane_addr + k * 16, xv[k]);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < kNpad / 16; ++k) tmem_regs_ready(xv[k]);
                if (kFp8) {
                    // x = (s_x s_w) * accumulator + bias
                    const float sc = *p.act_scale * p.w_scale;
#pragma unroll
                    for (int k = 0; k < kNpad / 16; ++k)
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            xv[k][e] = __float_as_uint(fmaf(__uint_as_float(xv[k][e]), sc, s_bias[k * 16 + e]));
                }
                if (h == 1) named_barrier_sync(4, 2 * kBM);  // group 0 is done with the tile
                // x^2 (bf16) into the 128-byte-swizzled operand tile
#pragma unroll
                for (int k = 0; k < kNpad / 16; ++k) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float a = __uint_as_float(xv[k][q * 8 + 2 * e]);
                            const float c = __uint_as_float(xv[k][q * 8 + 2 * e + 1]);
                            w[e] = pack_bf16x2(a * a, c * c);
                        }
                        const int k0 = k * 16 + q * 8;
                        const int kb = k0 / kBK, chunk = (k0 % kBK) / 8;
                        st_shared_v4(x2 + kb * (kBM * 128) + m * 128 + ((chunk ^ (m & 7)) << 4), w[0], w[1], w[2],
                                     w[3]);
                    }
                }
                fence_proxy_async_smem();
                tc_fence_before();  // the TMEM loads above precede the GEMM that overwrites those columns
                named_barrier_sync(1 + h, kBM);
                if (hleader) {
                    tc_fence_after();
                    const uint32_t g0 = smem_u32(smem + Lay::offG);
                    const uint32_t idesc = idesc_bf16(kBM, kNpad);
                    // norm = beta (ones x beta) + x^2 gamma^T, over this half's conv outputs
                    mma_bf16(dcol, smem_desc(smem_u32(smem + Lay::offOnes), 128, 256, 0),
                             smem_desc(smem_u32(smem + Lay::offBetaB), 128, 256, 0), idesc, 0);
#pragma unroll
                    for (int kk = 0; kk < kNpad / 16; ++kk) {
                        const uint32_t koff = (kk / 4) * (kBM * 128) + (kk % 4) * 32;
                        const uint32_t goff = (kk / 4) * (kNpad * 128) + (kk % 4) * 32;
                        mma_bf16(dcol, smem_desc(x2 + koff, 16, 1024, 2), smem_desc(g0 + goff, 16, 1024, 2), idesc, 1);
                    }
                    mma_commit(&g2bar[h]);
                    const bool ok = mbar_wait(&g2bar[h], j & 1, abort, kWaitNs);
                    if (!ok) fail(p, abort, kErrEpilogue);
                    *h_ok = ok ? 1 : 0;
                }
                named_barrier_sync(1 + h, kBM);
                const bool hok = *h_ok != 0;
                tc_fence_after();
                if (hok) {
                    // y = x * rsqrt(norm) (IGDN: x * sqrt(norm)) into the staging tile
                    // (the GEMM has read x^2), or straight to global memory
                    const int row = h * kBM + m;
                    const int ty = row / p.TX, tx = row - ty * p.TX;
                    const int gy = gy0 + ty, gx = gx0 + tx;
                    const bool valid = gy < p.GH && gx < p.GW;
                    const int oy = gy * p.out_step + (p.phases == 4 ? (ph >> 1) : 0);
                    const int ox = gx * p.out_step + (p.phases == 4 ? (ph & 1) : 0);
                    __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                          (((int64_t)b * p.Hout + oy) * p.Wout + ox) * kNpad;
                    uint32_t nv[2][16];
                    tmem_ld16(dcol + lane_addr, nv[0]);
#pragma unroll
                    for (int k = 0; k < kNpad / 16; ++k) {
                        tmem_wait_ld();
                        tmem_regs_ready(nv[k & 1]);
                        if (k + 1 < kNpad / 16) tmem_ld16(dcol + lane_addr + (k + 1) * 16, nv[(k + 1) & 1]);
                        uint32_t o[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float n0 = __uint_as_float(nv[k & 1][2 * e]);
                            const float n1 = __uint_as_float(nv[k & 1][2 * e + 1]);
                            const float r0 = kEpi == kEpiIgdn ? sqrt_approx(n0) : rsqrt_approx(n0);
                            const float r1 = kEpi == kEpiIgdn ? sqrt_approx(n1) : rsqrt_approx(n1);
                            o[e] = pack_bf16x2(__uint_as_float(xv[k][2 * e]) * r0, __uint_as_float(xv[k][2 * e + 1]) * r1);
                            if (valid) am2 = amax_bf16x2(am2, o[e]);
                        }
                        if (p.tma_store) {
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int k0 = k * 16 + q * 8;
                                const int kb = k0 / kBK, chunk = (k0 % kBK) / 8;
                                st_shared_v4(x2 + kb * (kBM * 128) + m * 128 + ((chunk ^ (m & 7)) << 4), o[q * 4],
                                             o[q * 4 + 1], o[q * 4 + 2], o[q * 4 + 3]);
                            }
                        } else if (valid) {
                            uint4 *dst = reinterpret_cast<uint4 *>(orow + k * 16);
                            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                }
                fence_proxy_async_smem();
                named_barrier_sync(1 + h, kBM);
                if (hleader && hok && p.tma_store) {
                    // this half: TY / 2 rows of the tile, 64 channels per box
                    const unsigned char *stg = smem + Lay::offX2;
                    const int hy = gy0 + h * (p.TY / 2);
                    if (p.tma_store == 2) {
                        const int yrow = b * p.GH + hy;
                        for (int kb = 0; kb < kNpad / kBK; ++kb)
                            tma_store_5d(&tmO, stg + kb * (kBM * 128), kb * kBK, ph & 1, gx0, ph >> 1, yrow);
                    } else {
                        for (int kb = 0; kb < kNpad / kBK; ++kb)
                            tma_store_4d(&tmO, stg + kb * (kBM * 128), kb * kBK, gx0, hy, b);
                    }
                    bulk_commit_group();
                }
                tc_fence_before();
                mbar_arrive(&acce[buf]);  // this thread is done with the accumulator
                if (hleader && p.tma_store) bulk_wait_read_all();  // the staging tile may be rewritten
                if (h == 0) named_barrier_arrive(4, 2 * kBM);
            }
            if (hleader && p.tma_store) bulk_wait_all();  // stores complete before the CTA exits
            if (p.amax_out) amax_flush(p.amax_out, am2);
        } else {
        // Warp w reads TMEM lanes 32*(w%4).. (tile rows); with 8 warps either
        // column half w/4 of every tile, or (ping-pong) all columns of the
        // tiles of group w/4.  A group's first thread alone waits on the
        // mbarriers and publishes the outcome in its epi_ok slot; the group
        // then meets at its named barrier, so it always takes the same branch
        // and no thread waits at a barrier the others have left.
        const int m = threadIdx.x & 127;  // TMEM lane = tile row = output pixel
        const int grp = Lay::kPingPong ? (warp >> 2) : 0;           // ping-pong group
        const bool gleader = (threadIdx.x & (Lay::kGroupThreads - 1)) == 0;
        const uint32_t gbar = 1 + grp;                               // the group's named barrier
        const int half = Lay::kPingPong ? 0 : (threadIdx.x >> 7);
        const int c_lo = half ? Lay::kSplit : 0, c_hi = half ? kNpad : Lay::kSplit;
        // GDN passes: columns per thread, equal for both halves, in 16-column chunks
        constexpr int kEpiChunks = (Lay::kEpiWarps == 8 ? Lay::kSplit : kNpad) / 16;
        static_assert(!kNorm || Lay::kEpiWarps != 8 || Lay::kPingPong || 2 * Lay::kSplit == kNpad,
                      "equal column halves");
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        bool consts = !kNorm;
        volatile int *g_ok = epi_ok + grp;
        uint32_t am2 = 0;  // max |output| of this thread's valid pixels (amax_out)
        uint64_t *g2 = &g2bar[grp];
        const uint32_t x2 = smem_u32(smem + Lay::offX2 + grp * Lay::kX2One);
        int j = grp;   // this CTA's tile index (groups take alternate tiles)
        int gj = 0;    // the group's own tile count (phase of its GDN barrier)
        for (int tile = unit0 + grp * unit_step; tile < p.tiles_total;
             tile += Lay::kGroups * unit_step, j += Lay::kGroups, ++gj) {
            int b, ph, gy0, gx0;
            tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
            gx0 += sub_x;
            const int buf = j % Lay::kAccBufs;
            const uint32_t use = j / Lay::kAccBufs;
            if (gleader) {
                // the x^2 tile doubles as the previous tile's output staging
                if (kNorm && p.tma_store) bulk_wait_read_all();
                bool ok = !*abort;
                if (ok && !consts) ok = mbar_wait(cbar, 0, abort, kWaitNs);
                if (ok) ok = mbar_wait(&accf[buf], use & 1, abort, kWaitNs);
                if (!ok) fail(p, abort, kErrEpilogue);
                *g_ok = ok ? 1 : 0;
            }
            named_barrier_sync(gbar, Lay::kGroupThreads);
            if (!*g_ok) break;
            consts = true;
            tc_fence_after();
            const int gy = gy0 + m / p.TX, gx = gx0 + m % p.TX;
            const bool valid = gy < p.GH && gx < p.GW;
            const int oy = gy * p.out_step + (p.phases == 4 ? (ph >> 1) : 0);
            const int ox = gx * p.out_step + (p.phases == 4 ? (ph & 1) : 0);
            const uint32_t d1 = tmem_base + buf * p.buf_stride + lane_addr;
            const float sc = kFp8 ? *p.act_scale * p.w_scale : 1.f;  // FP8: the operand scales
            if (kEpi == kEpiScatter) {
                // Transposed conv with few output channels: row m (an input
                // pixel of the 8 x 16 tile incl. a 1-pixel halo) holds its
                // contribution to all 25 taps x 3 outputs.  Each output pixel
                // of the 12 x 28 core block sums the 4-9 contributions that
                // land on it.
                const uint32_t S = smem_u32(smem + Lay::offS + grp * Lay::kSOne);
                {
                    constexpr int kChunks = kNpad / 16;
                    uint32_t v[kChunks][16];
#pragma unroll
                    for (int c = 0; c < kChunks; ++c) tmem_ld16(d1 + c * 16, v[c]);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < kChunks; ++c) tmem_regs_ready(v[c]);
                    // column 3 k + o = tap k, output o
#pragma unroll
                    for (int k = 0; k < 25; ++k) {
                        constexpr int kO = kScatterCout;
                        st_shared_v4(S + (m * Lay::kSRow + k * 4) * 4, v[(kO * k) / 16][(kO * k) % 16],
                                     v[(kO * k + 1) / 16][(kO * k + 1) % 16], v[(kO * k + 2) / 16][(kO * k + 2) % 16],
                                     0u);
                    }
                }
                named_barrier_sync(gbar, Lay::kGroupThreads);
                // One thread per core pixel (ci, cj): its 2 x 2 output pixels
                // (phase py, px) sum the taps ky = py, py + 2, .. and kx = px,
                // px + 2, .. of input pixel (ci + 1 + dr, cj + 1 + dc) with
                // dr = 1 - (ky - py) / 2, dc = 1 - (kx - px) / 2: every offset
                // is a constant, each tap one 16-byte load.  Taps are added
                // in ky-major order, as the 4-9 terms of each output pixel.
                const int t = threadIdx.x & (Lay::kGroupThreads - 1);
                if (t < kScatterCoreH * kScatterCoreW) {
                    const int ci = t / kScatterCoreW, cj = t - ci * kScatterCoreW;
                    const uint32_t sb = S + (((ci + 1) * kScatterTX + cj + 1) * Lay::kSRow) * 4;
                    float acc[2][2][kScatterCout];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int o = 0; o < kScatterCout; ++o) acc[q >> 1][q & 1][o] = s_bias[o];
#pragma unroll
                    for (int ky = 0; ky < 5; ++ky) {
#pragma unroll
                        for (int kx = 0; kx < 5; ++kx) {
                            const int dr = (2 - ky + (ky & 1)) >> 1, dc = (2 - kx + (kx & 1)) >> 1;
                            const float4 q =
                                ld_shared_v4f(sb + ((dr * kScatterTX + dc) * Lay::kSRow + (ky * 5 + kx) * 4) * 4);
                            float *a = acc[ky & 1][kx & 1];
                            a[0] += q.x;
                            a[1] += q.y;
                            a[2] += q.z;
                        }
                    }
                    float *out = reinterpret_cast<float *>(p.out);
                    const int64_t plane = (int64_t)p.Hout * p.Wout;
                    const int oy0 = 2 * (gy0 + ci), ox0 = 2 * (gx0 + cj);
                    // 8-byte pairs when every row starts 8-byte aligned
                    const bool pair = ox0 + 1 < p.Wout && (p.Wout & 1) == 0;
#pragma unroll
                    for (int py = 0; py < 2; ++py) {
                        const int oyv = oy0 + py;
                        if (oyv >= p.Hout || ox0 >= p.Wout) continue;
#pragma unroll
                        for (int o = 0; o < kScatterCout; ++o) {
                            float y0 = acc[py][0][o], y1 = acc[py][1][o];
                            if (p.clamp) {
                                y0 = fminf(fmaxf(y0, 0.f), 1.f);
                                y1 = fminf(fmaxf(y1, 0.f), 1.f);
                            }
                            float *dst = out + ((int64_t)b * kScatterCout + o) * plane + (int64_t)oyv * p.Wout + ox0;
                            if (pair) {
                                *reinterpret_cast<float2 *>(dst) = make_float2(y0, y1);
                            } else {
                                dst[0] = y0;
                                if (ox0 + 1 < p.Wout) dst[1] = y1;
                            }
                        }
                    }
                }
                named_barrier_sync(gbar, Lay::kGroupThreads);  // S is rewritten by the next tile
            } else if (kNorm) {
                // pass 1: x^2 (bf16) into the 128-byte-swizzled operand tile.
                // kXReg: the thread's columns all load at once and stay in
                // registers (the GDN GEMM then overwrites them in TMEM).
                // Otherwise 16-column chunks, the next chunk's TMEM load in
                // flight while this one is converted and stored.
                uint32_t xv[Lay::kXReg ? kEpiChunks : 1][16];
                if constexpr (Lay::kXReg) {
#pragma unroll
                    for (int k = 0; k < kEpiChunks; ++k) tmem_ld16(d1 + c_lo + k * 16, xv[k]);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < kEpiChunks; ++k) tmem_regs_ready(xv[k]);
                    if (kFp8) {  // x = (s_x s_w) * accumulator + bias
#pragma unroll
                        for (int k = 0; k < kEpiChunks; ++k)
#pragma unroll
                            for (int e = 0; e < 16; ++e)
                                xv[k][e] = __float_as_uint(fmaf(__uint_as_float(xv[k][e]), sc, s_bias[c_lo + k * 16 + e]));
                    }
#pragma unroll
                    for (int k = 0; k < kEpiChunks; ++k) {
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a = __uint_as_float(xv[k][q * 8 + 2 * e]);
                                const float bb = __uint_as_float(xv[k][q * 8 + 2 * e + 1]);
                                w[e] = pack_bf16x2(a * a, bb * bb);
                            }
                            const int k0 = c_lo + k * 16 + q * 8;
                            const int kb = k0 / kBK, chunk = (k0 % kBK) / 8;
                            st_shared_v4(x2 + kb * (kBM * 128) + m * 128 + ((chunk ^ (m & 7)) << 4), w[0], w[1], w[2],
                                         w[3]);
                        }
                    }
                    tc_fence_before();  // the TMEM loads above precede the GEMM that overwrites those columns
                } else {
                    uint32_t v[2][16];
                    tmem_ld16(d1 + c_lo, v[0]);
#pragma unroll
                    for (int k = 0; k < kEpiChunks; ++k) {
                        tmem_wait_ld();
                        tmem_regs_ready(v[k & 1]);
                        if (k + 1 < kEpiChunks) tmem_ld16(d1 + c_lo + (k + 1) * 16, v[(k + 1) & 1]);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                float a = __uint_as_float(v[k & 1][q * 8 + e * 2]);
                                float bb = __uint_as_float(v[k & 1][q * 8 + e * 2 + 1]);
                                if (kFp8) {  // x = (s_x s_w) * accumulator + bias
                                    const int c = c_lo + k * 16 + q * 8 + e * 2;
                                    a = fmaf(a, sc, s_bias[c]);
                                    bb = fmaf(bb, sc, s_bias[c + 1]);
                                }
                                w[e] = pack_bf16x2(a * a, bb * bb);
                            }
                            const int k0 = c_lo + k * 16 + q * 8;
                            const int kb = k0 / kBK, chunk = (k0 % kBK) / 8;
                            st_shared_v4(x2 + kb * (kBM * 128) + m * 128 + ((chunk ^ (m & 7)) << 4), w[0], w[1], w[2],
                                         w[3]);
                        }
                    }
                }
                fence_proxy_async_smem();
                named_barrier_sync(gbar, Lay::kGroupThreads);
                if (gleader) {
                    const uint32_t g0 = smem_u32(smem + Lay::offG);
                    // the norm: over x (kXReg) or in the columns beside it
                    const uint32_t d2 = tmem_base + buf * p.buf_stride + (Lay::kXReg ? 0 : kNpad);
                    bool ok = true;
                    if (kPair) {
                        // norm = x^2 (each CTA its 128 rows) x gamma^T (each CTA half
                        // the rows): the leader issues it once both tiles are written
                        mbar_arrive_cluster(mapa_shared(smem_u32(x2full), 0));
                        if (leader) {
                            ok = mbar_wait(x2full, j & 1, abort, kWaitNs, true);
                            if (ok) {
                                tc_fence_after();
                                const uint32_t idesc = idesc_bf16(2 * kBM, kNpad);
                                // norm = beta (ones x beta) + x^2 gamma^T
                                mma_bf16_pair(d2, smem_desc(smem_u32(smem + Lay::offOnes), 128, 256, 0),
                                              smem_desc(smem_u32(smem + Lay::offBetaB), 128, 256, 0), idesc, 0);
#pragma unroll
                                for (int kk = 0; kk < kNpad / 16; ++kk) {
                                    const uint32_t koff = (kk / 4) * (kBM * 128) + (kk % 4) * 32;
                                    const uint32_t goff = (kk / 4) * (Lay::kNB * 128) + (kk % 4) * 32;
                                    mma_bf16_pair(d2, smem_desc(x2 + koff, 16, 1024, 2),
                                                  smem_desc(g0 + goff, 16, 1024, 2), idesc, 1);
                                }
                                mma_commit_pair_both(g2, 3);
                            }
                        }
                    } else {
                        tc_fence_after();
                        const uint32_t idesc = idesc_bf16(kBM, kNpad);
                        // norm = beta (ones x beta) + x^2 gamma^T
                        mma_bf16(d2, smem_desc(smem_u32(smem + Lay::offOnes), 128, 256, 0),
                                 smem_desc(smem_u32(smem + Lay::offBetaB), 128, 256, 0), idesc, 0);
#pragma unroll
                        for (int kk = 0; kk < kNpad / 16; ++kk) {
                            const uint32_t koff = (kk / 4) * (kBM * 128) + (kk % 4) * 32;
                            const uint32_t goff = (kk / 4) * (kNpad * 128) + (kk % 4) * 32;
                            mma_bf16(d2, smem_desc(x2 + koff, 16, 1024, 2), smem_desc(g0 + goff, 16, 1024, 2), idesc,
                                     1);
                        }
                        mma_commit(g2);
                    }
                    if (ok) ok = mbar_wait(g2, gj & 1, abort, kWaitNs);
                    if (!ok) fail(p, abort, kErrEpilogue);
                    *g_ok = ok ? 1 : 0;
                }
                named_barrier_sync(gbar, Lay::kGroupThreads);
                if (!*g_ok) break;
                tc_fence_after();
                // pass 2: y = x * rsqrt(beta + norm)  (IGDN: x * sqrt(beta + norm)),
                // pipelined like pass 1 (kXReg: x from registers, the norm
                // from the columns x was in)
                __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                      (((int64_t)b * p.Hout + oy) * p.Wout + ox) * kNpad;
                {
                    constexpr uint32_t kNormCol = Lay::kXReg ? 0 : kNpad;
                    uint32_t v[2][16], nv[2][16];
                    if (!Lay::kXReg) tmem_ld16(d1 + c_lo, v[0]);
                    tmem_ld16(d1 + kNormCol + c_lo, nv[0]);
#pragma unroll
                    for (int k = 0; k < kEpiChunks; ++k) {
                        tmem_wait_ld();
                        if (!Lay::kXReg) tmem_regs_ready(v[k & 1]);
                        tmem_regs_ready(nv[k & 1]);
                        if (k + 1 < kEpiChunks) {
                            if (!Lay::kXReg) tmem_ld16(d1 + c_lo + (k + 1) * 16, v[(k + 1) & 1]);
                            tmem_ld16(d1 + kNormCol + c_lo + (k + 1) * 16, nv[(k + 1) & 1]);
                        }
                        const int c0 = c_lo + k * 16;
                        uint32_t o[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float n0 = __uint_as_float(nv[k & 1][2 * e]);
                            const float n1 = __uint_as_float(nv[k & 1][2 * e + 1]);
                            // GDN: x / sqrt(n); IGDN: x * sqrt(n)
                            const float r0 = kEpi == kEpiIgdn ? sqrt_approx(n0) : rsqrt_approx(n0);
                            const float r1 = kEpi == kEpiIgdn ? sqrt_approx(n1) : rsqrt_approx(n1);
                            float x0, x1;
                            if constexpr (Lay::kXReg) {  // scaled in pass 1
                                x0 = __uint_as_float(xv[k][2 * e]);
                                x1 = __uint_as_float(xv[k][2 * e + 1]);
                            } else {
                                x0 = __uint_as_float(v[k & 1][2 * e]);
                                x1 = __uint_as_float(v[k & 1][2 * e + 1]);
                                if (kFp8) {
                                    x0 = fmaf(x0, sc, s_bias[c0 + 2 * e]);
                                    x1 = fmaf(x1, sc, s_bias[c0 + 2 * e + 1]);
                                }
                            }
                            o[e] = pack_bf16x2(x0 * r0, x1 * r1);
                            if (valid) am2 = amax_bf16x2(am2, o[e]);
                        }
                        if (p.tma_store) {
                            // into the staging tile (the x^2 tile's layout: 128-byte
                            // rows per 64 channels, 16-byte chunks swizzled by row)
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int k0 = c0 + q * 8;
                                const int kb = k0 / kBK, chunk = (k0 % kBK) / 8;
                                st_shared_v4(x2 + kb * (kBM * 128) + m * 128 + ((chunk ^ (m & 7)) << 4), o[q * 4],
                                             o[q * 4 + 1], o[q * 4 + 2], o[q * 4 + 3]);
                            }
                        } else if (valid) {
                            uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
                            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                }
                if (p.tma_store) {
                    // the whole tile, 64 channels per box; TMA leaves out the
                    // pixels beyond the image
                    fence_proxy_async_smem();
                    named_barrier_sync(gbar, Lay::kGroupThreads);
                    if (gleader) {
                        const unsigned char *stg = smem + Lay::offX2 + grp * Lay::kX2One;
                        if (p.tma_store == 2) {
                            // transposed conv: phase (py, px) of the output viewed as
                            // [B * Hout / 2][py][Wout / 2][px][C]
                            const int yrow = b * p.GH + gy0;
                            for (int kb = 0; kb < kNpad / kBK; ++kb)
                                tma_store_5d(&tmO, stg + kb * (kBM * 128), kb * kBK, ph & 1, gx0, ph >> 1, yrow);
                        } else {
                            for (int kb = 0; kb < kNpad / kBK; ++kb)
                                tma_store_4d(&tmO, stg + kb * (kBM * 128), kb * kBK, gx0, gy0, b);
                        }
                        bulk_commit_group();
                    }
                }
            } else if (kEpi == kEpiBf16) {
                __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                      (((int64_t)b * p.Hout + oy) * p.Wout + ox) * kNpad;
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(d1 + c0, v);
                    tmem_wait_ld();
                    uint32_t o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        o[e] = kFp8 ? pack_bf16x2(fmaf(__uint_as_float(v[2 * e]), sc, s_bias[c0 + 2 * e]),
                                                  fmaf(__uint_as_float(v[2 * e + 1]), sc, s_bias[c0 + 2 * e + 1]))
                                    : pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
                    if (valid)
#pragma unroll
                        for (int e = 0; e < 8; ++e) am2 = amax_bf16x2(am2, o[e]);
                    if (valid) {
                        uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
                        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                    }
                }
            } else {
                // fp32 NCHW: per channel the warp's 32 pixels are contiguous in x
                float *out = reinterpret_cast<float *>(p.out);
                const int64_t plane = (int64_t)p.Hout * p.Wout;
                const int64_t pix = (int64_t)oy * p.Wout + ox;
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(d1 + c0, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int c = c0 + e;
                        float y = __uint_as_float(v[e]);
                        if (kFp8) y = fmaf(y, sc, s_bias[c]);
                        if (kEpi == kEpiF32Clamp) y = fminf(fmaxf(y, 0.f), 1.f);
                        if (valid && c < p.cout) out[((int64_t)b * p.cout_total + p.out_c0 + c) * plane + pix] = y;
                    }
                }
            }
            tc_fence_before();
            if (kPair) {
                // every epilogue thread of this CTA is done with the buffer; one
                // arrival per CTA on the leader's acce
                named_barrier_sync(gbar, Lay::kGroupThreads);
                if (gleader) mbar_arrive_cluster(mapa_shared(smem_u32(&acce[buf]), 0));
            } else {
                mbar_arrive(&acce[buf]);
            }
            // the next tile's epi_ok must not be written before every thread read this one
            named_barrier_sync(gbar, Lay::kGroupThreads);
        }
        if (kNorm && p.tma_store && gleader) bulk_wait_all();  // stores complete before the CTA exits
        if (p.amax_out) amax_flush(p.amax_out, am2);
        }
    } else if (kGather) {
        // ------------------------------------------------------------ gather (first layer)
        const int m = threadIdx.x - kGatherThread0;
        const uint32_t row_off = (m & 7) * 16 + (m >> 3) * 1280;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < p.tiles_total && !*abort; tile += gridDim.x, ++it) {
            int b, ph, gy0, gx0;
            tile_coords<kEpi == kEpiIgdn>(p, tile, b, ph, gy0, gx0);
            const int s = it % kStages;
            const uint32_t r = it / kStages;
            if (!mbar_wait(&empty[s], (r & 1) ^ 1, abort, kWaitNs)) {
                fail(p, abort, kErrGather);
                break;
            }
            const uint32_t a0 = smem_u32(smem + s * Lay::kStage) + row_off;
            if (p.patch_tma) {
                const int pb = (int)(it % Lay::kPatchBufs);
                if (!mbar_wait(&pfull[pb], (it / Lay::kPatchBufs) & 1, abort, kWaitNs)) {
                    fail(p, abort, kErrGather);
                    break;
                }
                // pixel (ty, tx) of the tile reads patch rows 2 ty + ky and
                // columns 2 tx + 2 + kx (the patch starts 2 rows above and 4
                // columns left of the tile's first output pixel's centre)
                const int ty = m / p.TX, tx = m - (m / p.TX) * p.TX;
                const float *pt = reinterpret_cast<const float *>(smem + Lay::offPatch + pb * kPatchBuf) +
                                  (2 * ty) * p.patch_w + 2 * tx + 2;
                float f[kGatherK];
#pragma unroll
                for (int ci = 0; ci < 3; ++ci) {
#pragma unroll
                    for (int ky = 0; ky < 5; ++ky) {
                        const float *q = pt + (ci * p.patch_h + ky) * p.patch_w;
                        const float2 v01 = *reinterpret_cast<const float2 *>(q);
                        const float2 v23 = *reinterpret_cast<const float2 *>(q + 2);
                        const int k = ci * 25 + ky * 5;
                        f[k] = v01.x;
                        f[k + 1] = v01.y;
                        f[k + 2] = v23.x;
                        f[k + 3] = v23.y;
                        f[k + 4] = q[4];
                    }
                }
#pragma unroll
                for (int k = 75; k < kGatherK; ++k) f[k] = 0.f;
#pragma unroll
                for (int kc = 0; kc < kGatherK / 8; ++kc)
                    st_shared_v4(a0 + kc * 128, pack_bf16x2(f[kc * 8], f[kc * 8 + 1]),
                                 pack_bf16x2(f[kc * 8 + 2], f[kc * 8 + 3]), pack_bf16x2(f[kc * 8 + 4], f[kc * 8 + 5]),
                                 pack_bf16x2(f[kc * 8 + 6], f[kc * 8 + 7]));
                mbar_arrive(&pempty[pb]);  // this thread has read the window
            } else {
            const int gy = gy0 + m / p.TX, gx = gx0 + m % p.TX;
            const bool valid = gy < p.GH && gx < p.GW;
            const float *img = p.x_in + (int64_t)b * 3 * p.Hin * p.Win;
#pragma unroll
            for (int kc = 0; kc < kGatherK / 8; ++kc) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int k = kc * 8 + e;
                    f[e] = 0.f;
                    if (k < 75) {
                        const int ci = k / 25, ky = (k % 25) / 5, kx = k % 5;
                        const int iy = 2 * gy + ky - 2, ix = 2 * gx + kx - 2;
                        if (valid && iy >= 0 && iy < p.Hin && ix >= 0 && ix < p.Win)
                            f[e] = __ldg(img + ((int64_t)ci * p.Hin + iy) * p.Win + ix);
                    }
                }
                st_shared_v4(a0 + kc * 128, pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                             pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
            }
            }
            fence_proxy_async_smem();
            mbar_arrive(&full[s]);
        }
    }

    // ---------------------------------------------------------------- teardown
    __syncthreads();
    if (*abort && leader) {
        // the two threads that issue MMAs (MMA lane, epilogue thread 0) commit
        // to dbar; TMEM is freed only once everything they issued completed
        if ((warp == kMmaWarp && lane == 0) || threadIdx.x == 0 ||
            ((Lay::kPingPong || Lay::kDual) && threadIdx.x == kBM)) {
            if (kPair) mma_commit_pair(dbar);
            else mma_commit(dbar);
        }
        if (warp == kMmaWarp && lane == 0) mbar_wait(dbar, 0, nullptr, kWaitNs / 10);
        __syncthreads();
    }
    // pairs: no remote arrive, load or MMA reaches a CTA that has left
    if (kPair) cluster_sync_all();
    if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        if (kPair) tmem_dealloc_pair(tmem_base, p.tmem_cols);
        else tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// bf16 operand tiles, 128-byte swizzled; fp32 = the first layer's unswizzled
// input windows.  Out-of-bounds elements read as zero.
enum class Elem { kBf16, kF32, kU8 };
static int make_map(CUtensorMap *map, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
                    const cuuint32_t *box, const cuuint32_t *estrides, bool fp32 = false, Elem elem = Elem::kBf16) {
    auto fn = encode_fn();
    if (!fn) return fcai::fail(FCAI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if (fp32) elem = Elem::kF32;
    const CUtensorMapDataType dt = elem == Elem::kF32  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : elem == Elem::kU8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = fn(map, dt, rank,
                    const_cast<void *>(base), dims, strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    fp32 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fcai::fail(FCAI_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return FCAI_OK;
}

// Largest power-of-two tile width (<= max_tx) that wastes the fewest columns.
static int pick_tx(int gw, int max_tx = 128) {
    int best = 8, waste_best = 1 << 30;
    for (int tx = 8; tx <= max_tx; tx <<= 1) {
        int waste = ((gw + tx - 1) / tx) * tx - gw;
        if (waste < waste_best || (waste == waste_best && tx > best)) {
            best = tx;
            waste_best = waste;
        }
    }
    return best;
}

template <int kNpad, int kEpi, bool kGather, bool kPair = false, bool kFp8 = false>
static int launch(const CUtensorMap &a, const CUtensorMap &w, const CUtensorMap &g, const CUtensorMap &o,
                  const ConvParams &p, cudaStream_t stream) {
    using Lay = Layout<kNpad, kEpi, kGather, kPair, kFp8>;
    static_assert(Lay::kAlloc <= kSmemBudget, "shared memory");
    auto kernel = conv_tc_kernel<kNpad, kEpi, kGather, kPair, kFp8>;
    static int configured[64] = {0};
    static int max_clusters[64] = {0};
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fcai::fail(FCAI_ERR_CUDA, "device ordinal %d unsupported", dev);
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(Lay::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Lay::kAlloc;
    cfg.stream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (!configured[dev]) {
        FCAI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc));
        if (kPair) {
            // pairs that can be resident at once (one CTA per SM)
            cfg.gridDim = dim3(2, 1, 1);
            int n = 0;
            FCAI_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
            if (n < 1) return fcai::fail(FCAI_ERR_CUDA, "no CTA pair of this layer fits on the device");
            max_clusters[dev] = n;
        }
        configured[dev] = 1;
    }
    if (kPair) {
        const int clusters = p.tiles_total < max_clusters[dev] ? p.tiles_total : max_clusters[dev];
        cfg.gridDim = dim3(2 * clusters, 1, 1);
        FCAI_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, a, w, g, o, p));
    } else {
        int grid = p.tiles_total < fcai::sm_count() ? p.tiles_total : fcai::sm_count();
        kernel<<<grid, Lay::kThreads, Lay::kAlloc, stream>>>(a, w, g, o, p);
    }
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

static int dispatch(int npad, int epi, bool gather, bool pair, bool fp8, const CUtensorMap &a, const CUtensorMap &w,
                    const CUtensorMap &g, const CUtensorMap &o, const ConvParams &p, cudaStream_t stream) {
    if (fp8) {
        if (npad == 128) {
            switch (epi) {
                case kEpiBf16: return launch<128, kEpiBf16, false, false, true>(a, w, g, o, p, stream);
                case kEpiGdn: return launch<128, kEpiGdn, false, false, true>(a, w, g, o, p, stream);
                case kEpiIgdn: return launch<128, kEpiIgdn, false, false, true>(a, w, g, o, p, stream);
                default: break;
            }
        } else if (npad == 192) {
            if (epi == kEpiF32) return launch<192, kEpiF32, false, false, true>(a, w, g, o, p, stream);
            if (epi == kEpiGdn) return launch<192, kEpiGdn, false, false, true>(a, w, g, o, p, stream);
            if (epi == kEpiIgdn) return launch<192, kEpiIgdn, false, false, true>(a, w, g, o, p, stream);
        } else if (npad == 160 && epi == kEpiF32) {
            return launch<160, kEpiF32, false, false, true>(a, w, g, o, p, stream);
        }
        return fcai::fail(FCAI_ERR_INVALID, "no FP8 kernel for npad=%d epilogue=%d", npad, epi);
    }
    if (pair) {
        if (npad == 128) {
            switch (epi) {
                case kEpiBf16: return launch<128, kEpiBf16, false, true>(a, w, g, o, p, stream);
                case kEpiGdn: return launch<128, kEpiGdn, false, true>(a, w, g, o, p, stream);
                case kEpiIgdn: return launch<128, kEpiIgdn, false, true>(a, w, g, o, p, stream);
                case kEpiF32: return launch<128, kEpiF32, false, true>(a, w, g, o, p, stream);
                default: break;
            }
        } else if (npad == 192) {
            if (epi == kEpiF32) return launch<192, kEpiF32, false, true>(a, w, g, o, p, stream);
            if (epi == kEpiBf16) return launch<192, kEpiBf16, false, true>(a, w, g, o, p, stream);
        }
        return fcai::fail(FCAI_ERR_INVALID, "no CTA-pair kernel for npad=%d epilogue=%d", npad, epi);
    }
    if (gather) {
        if (npad == 128 && epi == kEpiGdn) return launch<128, kEpiGdn, true>(a, w, g, o, p, stream);
        if (npad == 192 && epi == kEpiGdn) return launch<192, kEpiGdn, true>(a, w, g, o, p, stream);
        return fcai::fail(FCAI_ERR_INVALID, "first-layer kernel is built for 128 or 192 channels with GDN");
    }
    switch (npad) {
        case 128:
            switch (epi) {
                case kEpiBf16: return launch<128, kEpiBf16, false>(a, w, g, o, p, stream);
                case kEpiGdn: return launch<128, kEpiGdn, false>(a, w, g, o, p, stream);
                case kEpiIgdn: return launch<128, kEpiIgdn, false>(a, w, g, o, p, stream);
                case kEpiF32: return launch<128, kEpiF32, false>(a, w, g, o, p, stream);
                default: break;
            }
            break;
        case 192:
            if (epi == kEpiF32) return launch<192, kEpiF32, false>(a, w, g, o, p, stream);
            if (epi == kEpiBf16) return launch<192, kEpiBf16, false>(a, w, g, o, p, stream);
            if (epi == kEpiGdn) return launch<192, kEpiGdn, false>(a, w, g, o, p, stream);
            if (epi == kEpiIgdn) return launch<192, kEpiIgdn, false>(a, w, g, o, p, stream);
            break;
        case 160:  // half of a 320-channel latent layer
            if (epi == kEpiF32) return launch<160, kEpiF32, false>(a, w, g, o, p, stream);
            break;
        case 16:
            if (epi == kEpiF32Clamp) return launch<16, kEpiF32Clamp, false>(a, w, g, o, p, stream);
            if (epi == kEpiF32) return launch<16, kEpiF32, false>(a, w, g, o, p, stream);
            break;
        case 80:
            if (epi == kEpiScatter) return launch<80, kEpiScatter, false>(a, w, g, o, p, stream);
            break;
        default:
            break;
    }
    return fcai::fail(FCAI_ERR_INVALID, "no kernel instance for npad=%d epilogue=%d", npad, epi);
}

// Per-tensor e4m3 quantisation (the reference's _symmetric_scale and
// _quantize_fp8): amax of |x| over the tensor, scale = max(amax * fl(1/448), FLT_MIN),
// q = e4m3(clamp(x / scale, +-448)) rounded to nearest even.  |x| >= 0, so
// its float bits order like unsigned integers and atomicMax on them is the
// float maximum.
__global__ void amax_bf16_kernel(const uint4 *__restrict__ x, int64_t n8, uint32_t *amax_bits) {
    float m = 0.f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 v = x[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            m = fmaxf(m, fabsf(__uint_as_float(w[j] << 16)));
            m = fmaxf(m, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

// e4m3 code of one bf16 value x under the reference's rule (the scale as
// below): e4m3(clamp(x / scale, +-448)), x / scale a true division.  A NaN
// input divides to the GPU's canonical (positive) NaN, which torch.clamp
// passes through: code 0x7F whatever the input's sign.
__device__ __forceinline__ uint32_t e4m3_code(float x, float scale) {
    if (x != x) return 0x7Fu;
    float2 f;
    f.x = fminf(fmaxf(__fdiv_rn(x, scale), -448.f), 448.f);
    f.y = 0.f;
    return (uint32_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3) & 0xFFu;
}

// The output depends on the input's 16 bits alone, and the rule is odd in x
// (a negative x, -0 included, gives the code of |x| with the sign bit) but
// for NaN (0x7F, a code no number produces).  So
// each CTA first quantises the 32768 non-negative bf16 patterns into a
// shared-memory table with the same expression, then maps every element
// through it: one table read per element instead of a division, and the
// same bytes as quantising each element directly.
constexpr int kQuantThreads = 1024;
__global__ void __launch_bounds__(kQuantThreads) quantize_e4m3_kernel(const uint4 *__restrict__ x, uint2 *__restrict__ out,
                                                                      int64_t n8, const uint32_t *__restrict__ amax_bits,
                                                                      float *__restrict__ scale_out) {
    __shared__ uint8_t lut[32768];
    // the reference divides by the Python float 448, which PyTorch's CUDA
    // division by a host scalar computes as amax * fl(1 / 448); the elements
    // are then divided by the scale tensor (a true division)
    const float scale = fmaxf(__fmul_rn(__uint_as_float(*amax_bits), 1.0f / 448.0f), 1.17549435e-38f);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    for (int i = threadIdx.x; i < 32768; i += blockDim.x) lut[i] = (uint8_t)e4m3_code(__uint_as_float((uint32_t)i << 16), scale);
    __syncthreads();
    auto code = [&](uint32_t h) -> uint32_t {
        const uint32_t c = lut[h & 0x7FFFu];
        return c == 0x7Fu ? c : c | ((h >> 8) & 0x80u);
    };
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 v = x[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t q[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t a = w[2 * j], b = w[2 * j + 1];
            q[j] = code(a & 0xFFFFu) | (code(a >> 16) << 8) | (code(b & 0xFFFFu) << 16) | (code(b >> 16) << 24);
        }
        out[i] = make_uint2(q[0], q[1]);
    }
}

__global__ void nchw_to_nhwc_kernel(const float *__restrict__ in, __nv_bfloat16 *__restrict__ out, int C, int HW,
                                    int64_t total_pix) {
    // one thread per (pixel, 8-channel group): reads are strided by HW per
    // channel but coalesced across neighbouring pixels, writes are 16 bytes
    const int groups = C / 8;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total_pix * groups) return;
    const int g = (int)(idx / total_pix);
    const int64_t pix = idx - (int64_t)g * total_pix;
    const int64_t b = pix / HW, hw = pix - b * HW;
    const float *src = in + (b * C + g * 8) * HW + hw;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = pack_bf16x2(__ldg(src + (2 * e) * (int64_t)HW), __ldg(src + (2 * e + 1) * (int64_t)HW));
    *reinterpret_cast<uint4 *>(out + pix * C + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
}

// The same with 16 channels a thread where the channel count allows: the
// thread's two 16-byte stores fill one 32-byte sector of the pixel's NHWC
// row (rows of 16 k channels are 32-byte multiples), so no sector is written
// in halves by two threads far apart in time.
__global__ void nchw_to_nhwc16_kernel(const float *__restrict__ in, __nv_bfloat16 *__restrict__ out, int C, int HW,
                                      int64_t total_pix) {
    const int groups = C / 16;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total_pix * groups) return;
    const int g = (int)(idx / total_pix);
    const int64_t pix = idx - (int64_t)g * total_pix;
    const int64_t b = pix / HW, hw = pix - b * HW;
    const float *src = in + (b * C + g * 16) * HW + hw;
    uint32_t w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = pack_bf16x2(__ldg(src + (2 * e) * (int64_t)HW), __ldg(src + (2 * e + 1) * (int64_t)HW));
    uint4 *dst = reinterpret_cast<uint4 *>(out + pix * C + g * 16);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

}  // namespace ct

using namespace ct;

extern "C" {

int fcai_layer_out_size(const fcai_layer *L, int32_t h_in, int32_t w_in, int32_t *h_out, int32_t *w_out) {
    if (!L || !h_out || !w_out || h_in <= 0 || w_in <= 0) return fcai::fail(FCAI_ERR_INVALID, "invalid layer size query");
    if (L->kind == FCAI_LAYER_CONV5S2) {
        *h_out = (h_in + 4 - 5) / 2 + 1;
        *w_out = (w_in + 4 - 5) / 2 + 1;
    } else if (L->kind == FCAI_LAYER_DECONV5S2) {
        *h_out = 2 * h_in;
        *w_out = 2 * w_in;
    } else {
        return fcai::fail(FCAI_ERR_INVALID, "unknown layer kind %d", L->kind);
    }
    return FCAI_OK;
}

int fcai_layer_forward(const fcai_layer *L, int32_t batch, int32_t h_in, int32_t w_in, const void *input, void *output,
                       int32_t *err, fcai_stream_t stream_) {
    fcai::clear_error();
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!L || !input || !output || !L->weight || !L->bias) return fcai::fail(FCAI_ERR_INVALID, "null layer argument");
    int32_t ho, wo;
    int rc = fcai_layer_out_size(L, h_in, w_in, &ho, &wo);
    if (rc) return rc;
    if (batch <= 0 || batch > 65535) return fcai::fail(FCAI_ERR_INVALID, "batch out of range");
    const bool gather = L->in_format == FCAI_FMT_NCHW_F32;
    const bool deconv = L->kind == FCAI_LAYER_DECONV5S2;
    const int npad = L->npad;
    if (npad < L->cout || npad % 16 || npad > 256) return fcai::fail(FCAI_ERR_INVALID, "npad must round cout up to 16");
    if (gather && (deconv || L->cin != 3)) return fcai::fail(FCAI_ERR_INVALID, "fp32 NCHW input only for the cin=3 conv");
    if (!gather && L->cin % 64) return fcai::fail(FCAI_ERR_INVALID, "cin must be a multiple of 64");
    const bool norm = L->epilogue == FCAI_EPI_GDN || L->epilogue == FCAI_EPI_IGDN;
    if (norm && (!L->gdn_beta || !L->gdn_gamma || L->out_format != FCAI_FMT_NHWC_BF16))
        return fcai::fail(FCAI_ERR_INVALID, "GDN epilogue needs beta, gamma and a bf16 NHWC output");
    const bool scatter = L->algorithm == FCAI_ALGO_SCATTER;
    if (L->algorithm != FCAI_ALGO_IMPLICIT_GEMM && L->algorithm != FCAI_ALGO_SCATTER &&
        L->algorithm != FCAI_ALGO_IMPLICIT_GEMM_PAIR)
        return fcai::fail(FCAI_ERR_INVALID, "unknown layer algorithm %d", (int)L->algorithm);
    const bool pair = L->algorithm == FCAI_ALGO_IMPLICIT_GEMM_PAIR;
    // the kernel instance takes 256-pixel dual tiles exactly when this holds
    const bool dual = norm && !gather && !pair && npad <= 128;
    if (L->precision != FCAI_PREC_BF16 && L->precision != FCAI_PREC_FP8_E4M3)
        return fcai::fail(FCAI_ERR_INVALID, "unknown layer precision %d", (int)L->precision);
    const bool fp8 = L->precision == FCAI_PREC_FP8_E4M3;
    if (fp8) {
        if (gather || scatter || pair || L->cin % kBK)
            return fcai::fail(FCAI_ERR_INVALID,
                              "FP8 layers take e4m3 NHWC input with a multiple of 64 channels (no first-layer, "
                              "scatter or CTA-pair algorithm)");
        const bool f32_out = L->epilogue == FCAI_EPI_NONE && L->out_format == FCAI_FMT_NCHW_F32;
        if (!((npad == 128 && (L->epilogue != FCAI_EPI_NONE || L->out_format == FCAI_FMT_NHWC_BF16)) ||
              (npad == 192 && (norm || f32_out)) || (npad == 160 && f32_out)))
            return fcai::fail(FCAI_ERR_INVALID, "no FP8 kernel for npad=%d with this epilogue / output", npad);
        if (!L->act_scale || !(L->weight_scale > 0.f) || !(L->weight_scale < 3.0e38f))
            return fcai::fail(FCAI_ERR_INVALID, "FP8 layers need act_scale and a positive finite weight_scale");
        if (!L->bias) return fcai::fail(FCAI_ERR_INVALID, "FP8 layers need a bias");
    }
    if (pair && (gather || npad != L->cout || (npad != 128 && npad != 192)))
        return fcai::fail(FCAI_ERR_INVALID, "CTA-pair layers take bf16 NHWC input and 128 or 192 output channels");
    if (scatter && (!deconv || L->cout > 10 || npad != (25 * L->cout + 15) / 16 * 16 || norm ||
                    L->out_format != FCAI_FMT_NCHW_F32))
        return fcai::fail(FCAI_ERR_INVALID,
                          "scatter layers are transposed convolutions with cout <= 10, npad = round16(25 * cout) "
                          "and an fp32 NCHW output");
    if (scatter && L->cin > kScatterMaxCinBlocks * kBK)
        return fcai::fail(FCAI_ERR_INVALID, "scatter layers take at most %d input channels", kScatterMaxCinBlocks * kBK);
    int epi;
    if (scatter) epi = kEpiScatter;
    else if (L->epilogue == FCAI_EPI_GDN) epi = kEpiGdn;
    else if (L->epilogue == FCAI_EPI_IGDN) epi = kEpiIgdn;
    else if (L->out_format == FCAI_FMT_NHWC_BF16) epi = kEpiBf16;
    else epi = L->clamp01 ? kEpiF32Clamp : kEpiF32;

    ConvParams p{};
    p.B = batch;
    p.phases = deconv && !scatter ? 4 : 1;
    // phase-major tile order where the whole input is a small part of the
    // 126 MB L2 (every phase re-reads it; measured: it paid at 14 MB, g_s.0
    // at batch 24, and cost 1.6% at 38 MB, g_s.2)
    p.phase_major = p.phases == 4 && (int64_t)batch * h_in * w_in * L->cin * 2 <= (24ll << 20) ? 1 : 0;
    p.GH = deconv ? h_in : ho;
    p.GW = deconv ? w_in : wo;
    if (scatter) {
        // 8 x 16 input pixels per tile = a 6 x 14 core plus a 1-pixel halo;
        // the core produces a 12 x 28 output block
        p.TX = kScatterTX;
        p.TY = kScatterTY;
        p.step_x = kScatterCoreW;
        p.step_y = kScatterCoreH;
    } else {
        // the first layer's input windows come by TMA when the fp32 image
        // allows it: rows a multiple of 16 bytes, base 16-byte aligned
        const bool patch = gather && w_in % 4 == 0 && (reinterpret_cast<uintptr_t>(input) & 15) == 0;
        if (pair) {
            // a pair tile is two TX x TY sub-tiles side by side
            p.TX = pick_tx((p.GW + 1) / 2, 128);
            while (p.TX > 8 && ((p.GW + 2 * p.TX - 1) / (2 * p.TX)) * 2 * p.TX - p.GW >= p.TX) p.TX >>= 1;
        } else {
            p.TX = pick_tx(p.GW, patch ? kPatchMaxTX : 128);
        }
        p.TY = (dual ? 2 * kBM : kBM) / p.TX;
        p.step_x = pair ? 2 * p.TX : p.TX;
        p.step_y = p.TY;
        if (patch) {
            p.patch_tma = 1;
            p.patch_w = 2 * p.TX + 8;
            p.patch_h = 2 * p.TY + 3;
            p.patch_bytes = (uint32_t)(p.patch_w * p.patch_h * 3 * 4);
            if (p.patch_bytes > (uint32_t)kPatchBuf || p.patch_w > 256 || p.patch_h > 256)
                return fcai::fail(FCAI_ERR_INVALID, "first-layer input window exceeds its buffer");
        }
    }
    p.clamp = L->clamp01 ? 1 : 0;
    p.tiles_x = (p.GW + p.step_x - 1) / p.step_x;
    p.tiles_y = (p.GH + p.step_y - 1) / p.step_y;
    p.div_tx = make_fastdiv((uint32_t)p.tiles_x);
    p.div_ty = make_fastdiv((uint32_t)p.tiles_y);
    p.div_ph = make_fastdiv((uint32_t)p.phases);
    p.div_b = make_fastdiv((uint32_t)batch);
    p.stride = deconv ? 1 : 2;
    p.cin = L->cin;
    p.cout = L->cout;
    p.out_c0 = L->out_channel_offset;
    p.cout_total = L->out_channels_total ? L->out_channels_total : L->cout;
    if (p.out_c0 < 0 || p.out_c0 + p.cout > p.cout_total ||
        ((p.out_c0 || L->out_channels_total) && L->out_format != FCAI_FMT_NCHW_F32))
        return fcai::fail(FCAI_ERR_INVALID, "output channel range outside the fp32 NCHW output");
    // 128-byte K blocks.  FP8: 128 channels each; a last block past cin
    // (cin = 192, 320) reads as zeros (TMA fills elements outside the tensor)
    p.cin_blocks = gather ? 1 : (fp8 ? (L->cin + 2 * kBK - 1) / (2 * kBK) : L->cin / kBK);
    p.act_scale = fp8 ? L->act_scale : nullptr;
    if (L->amax_out && L->out_format != FCAI_FMT_NHWC_BF16)
        return fcai::fail(FCAI_ERR_INVALID, "amax_out is for layers with a bf16 NHWC output");
    if (L->amax_out && scatter) return fcai::fail(FCAI_ERR_INVALID, "amax_out is not produced by scatter layers");
    p.amax_out = L->amax_out;
    p.w_scale = fp8 ? L->weight_scale : 1.f;
    p.Hout = ho;
    p.Wout = wo;
    p.out_step = deconv ? 2 : 1;
    p.Hin = h_in;
    p.Win = w_in;
    const int64_t tiles = (int64_t)batch * p.phases * p.tiles_x * p.tiles_y;
    if (tiles > INT32_MAX) return fcai::fail(FCAI_ERR_INVALID, "too many tiles");
    p.tiles_total = (int)tiles;
    // GDN layers over 192 channels fed by TMA keep x in registers and write
    // the norm over it (npad columns a buffer); other GDN layers hold both
    const bool xreg = norm && npad > 128 && !gather;
    const int per_buf = npad + (norm && !xreg ? npad : 0);
    uint32_t stride = 32;
    while (stride < (uint32_t)per_buf) stride <<= 1;
    p.buf_stride = stride;
    // the kernel's accumulator buffer count (Layout::kAccBufs)
    p.tmem_cols = (scatter ? 4 : (norm && npad > 128 && gather ? 1 : 2)) * stride;
    if (p.tmem_cols > 512) return fcai::fail(FCAI_ERR_INVALID, "accumulators exceed tensor memory");
    if (scatter) {
        p.taps[0].n = 1;  // one K pass over the halo tile, all taps are GEMM columns
        p.taps[0].dy[0] = -1;
        p.taps[0].dx[0] = -1;
        p.taps[0].w[0] = 0;
    } else if (deconv) {
        for (int ph = 0; ph < 4; ++ph) {
            const int py = ph >> 1, px = ph & 1;
            int n = 0;
            for (int ky = py; ky < 5; ky += 2)
                for (int kx = px; kx < 5; kx += 2) {
                    p.taps[ph].dy[n] = (int8_t)((py + 2 - ky) / 2);
                    p.taps[ph].dx[n] = (int8_t)((px + 2 - kx) / 2);
                    p.taps[ph].w[n] = (uint8_t)(ky * 5 + kx);
                    ++n;
                }
            p.taps[ph].n = n;
        }
    } else {
        int n = 0;
        for (int ky = 0; ky < 5; ++ky)
            for (int kx = 0; kx < 5; ++kx) {
                p.taps[0].dy[n] = (int8_t)(ky - 2);
                p.taps[0].dx[n] = (int8_t)(kx - 2);
                p.taps[0].w[n] = (uint8_t)(ky * 5 + kx);
                ++n;
            }
        p.taps[0].n = n;
    }
    p.bias = L->bias;
    p.beta = L->gdn_beta;
    p.x_in = gather ? static_cast<const float *>(input) : nullptr;
    p.wgather = gather ? L->weight : nullptr;
    p.out = output;
    p.err = err;

    CUtensorMap ma{}, mw{}, mg{}, mo{};
    // GDN layers with bf16 NHWC output write through TMA stores (the output
    // base must be 16-byte aligned).  Conv: a tile's output pixels are a
    // dense 4-D box.  Transposed conv: phase (py, px) of the output is the
    // box [.., py, .., px, ..] of the 5-D view [B * Hout / 2][2][Wout / 2][2][C];
    // its row dimension runs across images, so it is used only when no tile
    // reaches past its image's last row (GH a multiple of TY).
    const bool store_ok = norm && L->out_format == FCAI_FMT_NHWC_BF16 && (reinterpret_cast<uintptr_t>(output) & 15) == 0;
    // dual tiles store each 128-row half on its own: TY / 2 rows
    const int box_rows = dual ? p.TY / 2 : p.TY;
    if (store_ok && !deconv) {
        p.tma_store = 1;
        cuuint64_t od[4] = {(cuuint64_t)npad, (cuuint64_t)wo, (cuuint64_t)ho, (cuuint64_t)batch};
        cuuint64_t os[3] = {(cuuint64_t)npad * 2, (cuuint64_t)wo * npad * 2, (cuuint64_t)ho * wo * npad * 2};
        cuuint32_t ob[4] = {(cuuint32_t)kBK, (cuuint32_t)p.TX, (cuuint32_t)box_rows, 1};
        cuuint32_t oe[4] = {1, 1, 1, 1};
        if ((rc = make_map(&mo, output, 4, od, os, ob, oe))) return rc;
    } else if (store_ok && deconv && p.GH % p.TY == 0 && ho == 2 * p.GH && wo == 2 * p.GW) {
        p.tma_store = 2;
        cuuint64_t od[5] = {(cuuint64_t)npad, 2, (cuuint64_t)p.GW, 2, (cuuint64_t)batch * p.GH};
        cuuint64_t os[4] = {(cuuint64_t)npad * 2, (cuuint64_t)2 * npad * 2, (cuuint64_t)wo * npad * 2,
                            (cuuint64_t)2 * wo * npad * 2};
        cuuint32_t ob[5] = {(cuuint32_t)kBK, 1, (cuuint32_t)p.TX, 1, (cuuint32_t)box_rows};
        cuuint32_t oe[5] = {1, 1, 1, 1, 1};
        if ((rc = make_map(&mo, output, 5, od, os, ob, oe))) return rc;
    }
    if (gather && p.patch_tma) {
        // fp32 NCHW image as [B][3][Hin][Win]; one box = one tile's window
        cuuint64_t dims[4] = {(cuuint64_t)w_in, (cuuint64_t)h_in, 3, (cuuint64_t)batch};
        cuuint64_t strides[3] = {(cuuint64_t)w_in * 4, (cuuint64_t)h_in * w_in * 4, (cuuint64_t)3 * h_in * w_in * 4};
        cuuint32_t box[4] = {(cuuint32_t)p.patch_w, (cuuint32_t)p.patch_h, 3, 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        if ((rc = make_map(&ma, input, 4, dims, strides, box, es, true))) return rc;
    }
    if (!gather) {
        // operands: bf16 (2 bytes) or e4m3 (1 byte) elements; one box row is
        // 128 bytes of channels either way
        const int s = p.stride;
        const cuuint64_t eb = fp8 ? 1 : 2;
        const cuuint32_t ke = fp8 ? 2 * kBK : kBK;
        const Elem el = fp8 ? Elem::kU8 : Elem::kBf16;
        cuuint64_t dims[4] = {(cuuint64_t)L->cin, (cuuint64_t)w_in, (cuuint64_t)h_in, (cuuint64_t)batch};
        cuuint64_t strides[3] = {(cuuint64_t)L->cin * eb, (cuuint64_t)w_in * L->cin * eb,
                                 (cuuint64_t)h_in * w_in * L->cin * eb};
        cuuint32_t box[4] = {ke, (cuuint32_t)(p.TX * s), (cuuint32_t)(p.TY * s), 1};
        cuuint32_t es[4] = {1, (cuuint32_t)s, (cuuint32_t)s, 1};
        if ((rc = make_map(&ma, input, 4, dims, strides, box, es, false, el))) return rc;
        cuuint64_t wd[3] = {(cuuint64_t)L->cin, (cuuint64_t)npad, (cuuint64_t)(scatter ? 1 : 25)};
        cuuint64_t ws[2] = {(cuuint64_t)L->cin * eb, (cuuint64_t)npad * L->cin * eb};
        cuuint32_t wb[3] = {ke, (cuuint32_t)(pair ? npad / 2 : npad), 1};  // pairs: half the rows each
        cuuint32_t we[3] = {1, 1, 1};
        if ((rc = make_map(&mw, L->weight, 3, wd, ws, wb, we, false, el))) return rc;
    }
    if (norm) {
        cuuint64_t gd[3] = {(cuuint64_t)npad, (cuuint64_t)npad, 1};
        cuuint64_t gs[2] = {(cuuint64_t)npad * 2, (cuuint64_t)npad * npad * 2};
        cuuint32_t gb[3] = {(cuuint32_t)kBK, (cuuint32_t)(pair ? npad / 2 : npad), 1};
        cuuint32_t ge[3] = {1, 1, 1};
        if ((rc = make_map(&mg, L->gdn_gamma, 3, gd, gs, gb, ge))) return rc;
    }
    return dispatch(npad, epi, gather, pair, fp8, ma, mw, mg, mo, p, stream);
}

int fcai_quantize_e4m3(const void *input_bf16, void *output_e4m3, float *scale_out, uint32_t *amax_work,
                       int32_t amax_ready, int64_t count, fcai_stream_t stream_) {
    fcai::clear_error();
    if (!input_bf16 || !output_e4m3 || !scale_out || !amax_work || count <= 0 || count % 8 ||
        (reinterpret_cast<uintptr_t>(input_bf16) & 15) || (reinterpret_cast<uintptr_t>(output_e4m3) & 7) ||
        (reinterpret_cast<uintptr_t>(amax_work) & 3) || (reinterpret_cast<uintptr_t>(scale_out) & 3))
        return fcai::fail(FCAI_ERR_INVALID, "invalid e4m3 quantisation arguments");
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    const int64_t n8 = count / 8;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((n8 + threads - 1) / threads, (int64_t)fcai::sm_count() * 8);
    if (!amax_ready) {
        FCAI_CUDA_TRY(cudaMemsetAsync(amax_work, 0, sizeof(uint32_t), stream));
        ct::amax_bf16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const uint4 *>(input_bf16), n8,
                                                                        amax_work);
        FCAI_CUDA_TRY(cudaGetLastError());
    }
    // one CTA of 1024 threads per SM (each builds its 32 KB table once),
    // fewer for small inputs
    const int64_t qblocks =
        std::min<int64_t>((n8 + ct::kQuantThreads - 1) / ct::kQuantThreads, (int64_t)fcai::sm_count());
    ct::quantize_e4m3_kernel<<<(unsigned)qblocks, ct::kQuantThreads, 0, stream>>>(
        static_cast<const uint4 *>(input_bf16), static_cast<uint2 *>(output_e4m3), n8, amax_work, scale_out);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

int fcai_nchw_f32_to_nhwc_bf16(const float *input, void *output, int32_t batch, int32_t channels, int32_t h, int32_t w,
                               fcai_stream_t stream_) {
    fcai::clear_error();
    if (!input || !output || batch <= 0 || channels <= 0 || channels % 8 || h <= 0 || w <= 0)
        return fcai::fail(FCAI_ERR_INVALID, "invalid layout conversion arguments");
    const int64_t pix = (int64_t)batch * h * w;
    const bool wide = channels % 16 == 0;
    const int64_t total = pix * (channels / (wide ? 16 : 8));
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    if (wide)
        nchw_to_nhwc16_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
            input, static_cast<__nv_bfloat16 *>(output), channels, h * w, pix);
    else
        nchw_to_nhwc_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
            input, static_cast<__nv_bfloat16 *>(output), channels, h * w, pix);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

}  // extern "C"
