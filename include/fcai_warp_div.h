/*
 * fcai_warp_div.h -- C ABI of the B200 `warp_div` entropy coder.
 *
 * This library replaces the reference's native module
 * `fast_compressai.coders._warp_div` (coders/cuda/ans_gpu.cpp:25-30), whose
 * two pybind entry points take and return torch tensors:
 *
 *   encode_warp_div(symbols, indexes, cdfs, cdf_sizes, offsets, P)
 *       -> (packed, max_rounds, header_bytes, chunk_len, P)
 *       coders/cuda/warp_ans_kernel_v2.cu:183-306
 *   decode_warp_div(packed, max_rounds, header_bytes, chunk_len, P,
 *                   indexes, cdfs, cdf_sizes, offsets) -> symbols
 *       coders/cuda/warp_ans_kernel.cu:477-544
 *
 * Here every buffer is a plain device pointer owned by the caller.  The
 * payload size is only known after encoding, so encode is split in two
 * calls: fcai_warp_div_encode() codes the symbols into the workspace and
 * reports the exact payload size (one small device-to-host read, the only
 * synchronisation of the encode path); fcai_warp_div_encode_pack() then
 * writes the payload into a buffer of exactly that size.
 *
 * Payload layout (bit-exact with the reference, little-endian u32 words):
 *   h0 = N, h1 = chunk_len, h2 = K | B << 16, h3 = 2 | 32 << 16,
 *   h4..h7 = 0, then int32 max_rounds[B*K] at byte 32, zero padding to a
 *   16-byte boundary (header_bytes), then for every chunk (b-major) its
 *   max_rounds x 32 interleaved words: word r of lane L at r*32 + L.
 *
 * All calls enqueue work on `stream` of the current CUDA device; the caller
 * selects the device.  Inputs are int32 and contiguous.  `indexes` may be
 * NULL, meaning the channel layout indexes[b, i] = i / (N / C) that
 * CompressAI's EntropyBottleneck builds; results are identical to passing
 * that tensor explicitly.
 *
 * Workspaces: the first 256 bytes of every workspace are a control block that
 * must be zero before its first use (e.g. cudaMemset); every call leaves it
 * zero again.  A workspace must not be used by two calls that can overlap on
 * the GPU.
 */
#ifndef FCAI_WARP_DIV_H
#define FCAI_WARP_DIV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *fcai_stream_t; /* a cudaStream_t; NULL = default stream */

/* Status codes.  Values 1..7 are caller errors that the Python layer maps
 * to CoderInputError, as the reference maps TORCH_CHECK failures
 * (coders/warp_div.py:101-102,148-149). */
enum {
    FCAI_OK = 0,
    FCAI_ERR_INVALID = 1,     /* bad argument, shape or size limit */
    FCAI_ERR_INDEX_RANGE = 2, /* an index outside [0, C) */
    FCAI_ERR_TABLE = 3,       /* cdf_size outside [2, L] or a row not strictly increasing in [0, 65536] */
    FCAI_ERR_HEADER = 4,      /* payload header words inconsistent with the metadata */
    FCAI_ERR_ROUNDS = 5,      /* header round table differs from max_rounds */
    FCAI_ERR_CORRUPT = 6,     /* payload length or body inconsistent with the rounds */
    FCAI_ERR_WORKSPACE = 7,   /* workspace smaller than the plan requires */
    FCAI_ERR_CUDA = 8         /* a CUDA runtime call failed */
};

/* Sizes derived from (B, N, C, P), as the reference host code derives them
 * (coders/cuda/warp_ans_kernel_v2.cu:216-279). */
typedef struct {
    int32_t chunks;                 /* K = ceil(C / P) */
    int32_t chunk_len;              /* P * (N / C) */
    int64_t header_bytes;           /* align16(32 + 4 * B * K) */
    int64_t encode_workspace_bytes; /* for fcai_warp_div_encode / _pack */
    int64_t decode_workspace_bytes; /* for fcai_warp_div_decode */
    int64_t max_packed_bytes;       /* worst-case payload size */
} fcai_warp_div_plan;

/* Checks the reference's size preconditions (warp_ans_kernel_v2.cu:198-203:
 * B, N, C > 0, N % C == 0, 1 <= P <= C, B and C <= 65535, N * C < 2^31 - 1)
 * and fills `plan`. */
int fcai_warp_div_plan_create(int32_t B, int32_t N, int32_t C, int32_t P, fcai_warp_div_plan *plan);

typedef struct {
    int64_t packed_bytes;           /* exact payload size for _pack */
    int64_t header_bytes;
    int64_t required_workspace_bytes; /* smallest workspace that holds this
                                         call's staging (set on success and
                                         on FCAI_ERR_WORKSPACE) */
    int32_t chunk_len;
    int32_t p_ch;
    int32_t index_layout_is_channel; /* 1 when indexes == channel layout (or NULL) */
    int32_t reserved;
} fcai_warp_div_encode_info;

/* Encode symbols[B,N] (replaces encode_with_indexes_warp_v2_cuda,
 * coders/cuda/warp_ans_kernel_v2.cu:183-306, up to the payload allocation).
 * Writes max_rounds[B*K] (uint32, device) and fills *info on the host.
 * Blocks the host until the size is known.  A workspace of
 * plan.encode_workspace_bytes always suffices; a smaller one works while the
 * lanes' words fit and otherwise returns FCAI_ERR_WORKSPACE with
 * info->required_workspace_bytes set, after which the call can be repeated
 * with a larger workspace. */
int fcai_warp_div_encode(const int32_t *symbols, const int32_t *indexes, int32_t B, int32_t N,
                         const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                         const int32_t *offsets, int32_t P, void *workspace, int64_t workspace_bytes,
                         uint32_t *max_rounds, fcai_warp_div_encode_info *info, fcai_stream_t stream);

/* Write the payload of the last fcai_warp_div_encode on this workspace into
 * packed[packed_bytes] (the header and pack steps, warp_ans_kernel.cu:178-213,
 * 343-369).  Asynchronous. */
int fcai_warp_div_encode_pack(const void *workspace, int64_t workspace_bytes, int32_t B, int32_t N, int32_t C,
                              int32_t P, uint8_t *packed, int64_t packed_bytes, fcai_stream_t stream);

/* Decode a payload into symbols_out[B,N] (replaces
 * decode_with_indexes_warp_cuda, coders/cuda/warp_ans_kernel.cu:477-544,
 * together with the header check of coders/warp_div.py:161-176).  K is
 * taken from max_rounds' shape as in the reference; the workspace needs
 * 256 + align256(8 * B * K) bytes.  With check != 0 the call waits for the
 * GPU and returns FCAI_ERR_HEADER / _ROUNDS / _CORRUPT / _INDEX_RANGE /
 * _TABLE when the payload or tables are inconsistent (symbols_out then
 * holds no result) and, if index_layout_is_channel is not NULL, stores
 * whether indexes equal the channel layout.  With check == 0 the call is
 * asynchronous and a bad payload leaves symbols_out unspecified. */
int fcai_warp_div_decode(const uint8_t *packed, int64_t packed_bytes, const uint32_t *max_rounds, int32_t K,
                         int64_t header_bytes, int32_t chunk_len, const int32_t *indexes, int32_t B, int32_t N,
                         const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                         const int32_t *offsets, int32_t *symbols_out, void *workspace, int64_t workspace_bytes,
                         int32_t check, int32_t *index_layout_is_channel, fcai_stream_t stream);

/* Encode straight from the fp32 latent y[B, C*H*W] of a FactorizedPrior:
 * symbol = (int32)rint(y - medians[c]) with the channel layout, which is
 * CompressAI's EntropyBottleneck.quantize(y, "symbols", medians) followed by
 * the reference codec's encode (coders/factorized.py:46-59) in one pass.
 * The payload equals fcai_warp_div_encode's for those symbols. */
int fcai_warp_div_encode_latent(const float *y, const float *medians, int32_t B, int32_t N, const int32_t *cdfs,
                                int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets, int32_t P,
                                void *workspace, int64_t workspace_bytes, uint32_t *max_rounds,
                                fcai_warp_div_encode_info *info, fcai_stream_t stream);

/* The encode of fcai_warp_div_encode_latent in two halves, so that the
 * host's wait for the payload size overlaps device work.  _submit enqueues
 * the encode (its last CTA writes the status words to the stream's mapped
 * pinned slot) and returns at once (same
 * arguments, no info); the caller may then enqueue other work on the stream
 * (the next batch's analysis transform, an earlier batch's decode).
 * _finish waits for the submitted encode alone, not for that later work,
 * and fills *info as fcai_warp_div_encode_latent does (FCAI_ERR_WORKSPACE
 * included: repeat the encode with the larger workspace).  One submitted
 * encode per stream at a time: until its _finish, any other encode on the
 * stream is refused (FCAI_ERR_INVALID).  The workspace and max_rounds stay
 * in use until the _finish and the _pack.  No counterpart in the
 * reference, whose encode always blocks (warp_ans_kernel_v2.cu:183-306). */
int fcai_warp_div_encode_latent_submit(const float *y, const float *medians, int32_t B, int32_t N,
                                       const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                                       const int32_t *offsets, int32_t P, void *workspace, int64_t workspace_bytes,
                                       uint32_t *max_rounds, fcai_stream_t stream);
int fcai_warp_div_encode_finish(int32_t B, int32_t N, int32_t C, int32_t P, int64_t workspace_bytes,
                                fcai_warp_div_encode_info *info, fcai_stream_t stream);

/* Encode without a caller workspace and without allocating: the work of
 * fcai_warp_div_encode followed by fcai_warp_div_encode_pack, with the
 * encode workspace taken from a static device array of
 * FCAI_WARP_DIV_SCRATCH_BYTES (16 MiB) that this library holds on each
 * device it runs on.  No counterpart in the reference, whose encode
 * allocates its staging and payload tensors on every call.
 *
 * Meant for callers that cannot allocate device memory on the encode path:
 * a host-language binding (cgo, JNI, ctypes) that holds device pointers but
 * no device allocator of its own; a process whose device memory is already
 * held by another allocator (a caching allocator that owns the GPU), where
 * a cudaMalloc would fail; and a stream of queued work that a cudaMalloc or
 * cudaFree would stall by synchronising the device.
 *
 * Limit: sizes whose worst-case workspace (plan.encode_workspace_bytes)
 * exceeds FCAI_WARP_DIV_SCRATCH_BYTES are rejected with FCAI_ERR_WORKSPACE
 * and info->required_workspace_bytes set; use fcai_warp_div_encode with a
 * workspace of that size instead.  The payload goes to packed (device,
 * packed_capacity bytes; plan.max_packed_bytes always suffices) and its
 * size to info->packed_bytes; FCAI_ERR_INVALID if it does not fit.  Writes
 * max_rounds[B*K] like fcai_warp_div_encode and blocks the host until the
 * size is known; the payload write is then asynchronous on `stream`.
 *
 * All calls on a device share the one array, which keeps the previous
 * call's contents; each call clears the part that must start at zero.
 * Calls whose GPU work overlaps (issued on different streams, or from
 * different threads, with nothing ordering them) race on the array and
 * corrupt each other's payloads: issue them on one stream or serialise
 * them.
 *
 * No call allocates: no cudaMalloc, cudaFree, cudaHostAlloc or event
 * creation, on the first call on a device or stream as on any other.  The
 * status words that size the payload come back by a cudaMemcpyAsync into
 * the call's own stack frame followed by a wait for `stream`.  The first
 * call on each device does a one-time set-up with that device current: it
 * looks up the array's device address (cudaGetSymbolAddress; under CUDA's
 * lazy module loading, the default, this is also when the array is
 * reserved in the device's memory), and, if no other coder call has run on
 * the device yet, fills the library's division table with one kernel and a
 * wait for `stream`.  Make that first call early, before another allocator
 * takes the device's memory (or run with CUDA_MODULE_LOADING=EAGER, which
 * reserves the array when the library's kernels load), and before any
 * stream capture.  The set-up is cached per device ordinal for the life of
 * the process: a cudaDeviceReset invalidates it, and is not supported while
 * this library is in use. */
#define FCAI_WARP_DIV_SCRATCH_BYTES (16 * 1024 * 1024)
int fcai_warp_div_encode_noalloc(const int32_t *symbols, const int32_t *indexes, int32_t B, int32_t N,
                                 const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                                 const int32_t *offsets, int32_t P, uint8_t *packed, int64_t packed_capacity,
                                 uint32_t *max_rounds, fcai_warp_div_encode_info *info, fcai_stream_t stream);

/* Decode straight to the fp32 dequantised latent y_hat = (float)symbol +
 * medians[c] (coders/factorized.py:90-101: decode, then
 * EntropyBottleneck.dequantize), channel layout. */
int fcai_warp_div_decode_latent(const uint8_t *packed, int64_t packed_bytes, const uint32_t *max_rounds, int32_t K,
                                int64_t header_bytes, int32_t chunk_len, int32_t B, int32_t N, const int32_t *cdfs,
                                int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets,
                                const float *medians, float *y_hat_out, void *workspace, int64_t workspace_bytes,
                                int32_t check, fcai_stream_t stream);

/* Copy `bytes` from src to dst on `stream` with SM loads and stores, where
 * each operand is memory of the current device or pinned host memory mapped
 * into its address space (cudaHostAlloc memory on a system with unified
 * addressing).  For moving a payload between host and device while a batch's
 * bulk copies occupy the copy engines: this copy does not queue behind them.
 * FCAI_ERR_INVALID if an operand is neither (nothing is launched then).
 * Asynchronous; the host memory must stay allocated until the stream passes
 * the copy.  No counterpart in the reference (its payload stays a device
 * tensor). */
int fcai_payload_copy_async(void *dst, const void *src, int64_t bytes, fcai_stream_t stream);

/* Message of the last error on the calling thread ("" if none). */
const char *fcai_last_error(void);

/* Library version string. */
const char *fcai_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FCAI_WARP_DIV_H */
