// warp_div.cu -- B200 (sm_100a) kernels of the `warp_div` rANS coder and the
// C ABI declared in include/fcai_warp_div.h.
//
// Format (fixed by the reference, coders/cuda/warp_ans_kernel*.cu): the B x N
// symbols of a batch are cut into K = ceil(C / P) chunks per image of
// chunk_len = P * (N / C) consecutive symbols.  Inside a chunk, lane L of 32
// owns symbols start + L, start + L + 32, ...  Each lane is an independent
// 64-bit rANS stream (L = 2^31, 32-bit renormalisation, 16-bit CDFs, 4-bit
// bypass escapes); its words are stored interleaved (word r of lane L at
// r*32 + L) and every chunk is padded to the longest lane (max_rounds).
//
// Design (B200-first, not a translation of the reference):
//  * encode (channel layout: the codec's latent path and NULL indexes) is one
//    persistent kernel, encode_lanes_kernel: a CTA stages one chunk group's
//    P CDF rows in shared memory as 16-byte entries {division magic, freq,
//    start}, and each warp codes one chunk of the group.  Symbols are read
//    8 ahead; a batch in one channel reads its entries before its coder
//    steps, and when no lane escapes and every lane has room each step is a
//    fixed sequence (predicated renormalisation store, one 64-bit high
//    multiply, a 32-bit remainder correction).  Renormalisation words go to
//    a staging area [chunk][emission j][lane]; the last CTA to finish
//    computes the chunk offsets (exclusive scan of max_rounds * 32) and a
//    status block, so the host needs one small device-to-host read to size
//    the payload.
//  * pack reads each chunk's staging rows in emission order (128-byte rows)
//    and writes every lane's words in decode order, plus the header.
//  * decode (channel layout) is one persistent kernel, decode_lanes_kernel:
//    the group's rows and a slot-bucket table (8-byte entries that resolve a
//    bucket of one or two symbols without a search) in shared memory; each
//    step reads one bucket entry, and the refill word is loaded one step
//    ahead so the refill is a register move.  A validation/scan kernel runs
//    first for payloads from elsewhere (header words, round table, length).
//  * explicit indexes use full-table kernels (every row of the batch staged
//    per CTA); rows that do not fit in shared memory are read from global
//    memory by fallback kernels.
//  * all reads of payload words are bounded by the chunk's rounds and by the
//    escape limit (<= 8 nibbles), so corrupt payloads raise an error
//    instead of reading out of bounds.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/fcai_warp_div.h"
#include "fcai_common.h"

namespace fcai {

static thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < 64 && cache[dev]) return cache[dev];
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev < 64) cache[dev] = n;
    return n;
}

}  // namespace fcai

namespace wd {

constexpr int kLanes = 32;
constexpr int kWarps = 8;                 // warps per CTA
constexpr int kThreads = kLanes * kWarps;
constexpr uint64_t kRansL = 1ull << 31;
constexpr uint32_t kBypassBits = 4;
constexpr uint32_t kBypassMax = 15;
constexpr int kLutShift = 9;              // decode LUT bucket = slot >> 9
constexpr int kLutBuckets = 65536 >> kLutShift;
constexpr int kMaxSymbolWords = 10;       // <= 8 nibbles + count + symbol puts
constexpr int64_t kCtrlBytes = 256;
constexpr int kMaxSmemBytes = 200 * 1024;

// Error flags (bit mask accumulated in the control block).
enum : uint32_t {
    kFlagIndexRange = 1u << 0,
    kFlagNonChannel = 1u << 1,  // informational: indexes differ from the channel layout
    kFlagTable = 1u << 2,
    kFlagOverflow = 1u << 3,
    kFlagHeader = 1u << 4,
    kFlagRounds = 1u << 5,
    kFlagCorrupt = 1u << 6,
};

struct Control {
    unsigned int done;      // CTAs finished (reset by the last one)
    unsigned int flags;     // OR of flags (reset by the last one)
    unsigned int max_used;  // longest lane in words (reset by the last one)
    unsigned int pad0;
    long long status[8];    // written by the last CTA, read by the host
    unsigned int pad1[44];
};
static_assert(sizeof(Control) <= kCtrlBytes, "control block too large");
// status[] slots
constexpr int kStTotalWords = 0, kStFlags = 1, kStMaxUsed = 2, kStRowsCap = 3;

__host__ __device__ inline int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

struct EncLayout {
    int64_t rounds, used, offsets, stage, fixed_bytes;
};

__host__ __device__ inline EncLayout enc_layout(int64_t chunks) {
    EncLayout l;
    l.rounds = kCtrlBytes;
    l.used = l.rounds + align256(chunks * 4);
    l.offsets = l.used + align256(chunks * kLanes * 4);
    l.stage = l.offsets + align256(chunks * 8);
    l.fixed_bytes = l.stage;
    return l;
}

struct DecLayout {
    int64_t offsets, fixed_bytes;
};

__host__ __device__ inline DecLayout dec_layout(int64_t chunks) {
    DecLayout l;
    l.offsets = kCtrlBytes;
    l.fixed_bytes = l.offsets + align256(chunks * 8);
    return l;
}

// floor((2^64 - 1) / f) for f in [2, 65536]; entries 0 and 1 unused.
__device__ uint64_t g_magic[65537];

__global__ void init_magic_kernel() {
    int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f <= 65536) g_magic[f] = f >= 1 ? (~0ull) / (uint64_t)f : 0ull;
}

// ---------------------------------------------------------------------------
// CDF tables
// ---------------------------------------------------------------------------

// Packed entry of symbol v of a row: start | (freq - 1) << 16.  Valid rows
// have 0 <= start <= 65535 and 1 <= freq <= 65536.
__device__ __forceinline__ uint32_t pack_entry(int32_t a, int32_t b, uint32_t &flags) {
    if (a < 0 || b <= a || b > 65536) {
        flags |= kFlagTable;
        return 0u;  // start 0, freq 1: keeps the coder in bounds
    }
    return (uint32_t)a | ((uint32_t)(b - a - 1) << 16);
}

struct TableArgs {
    const int32_t *__restrict__ cdfs;
    const int32_t *__restrict__ sizes;
    const int32_t *__restrict__ offs;
    int C, L;
};

// Stages every row into shared memory: entries [C][L-1] and {offset, maxv}.
// With lut != nullptr also builds the decode bucket table [C][kLutBuckets].
__device__ void stage_tables(const TableArgs &t, uint32_t *s_tab, int2 *s_ch, uint16_t *s_lut,
                             uint32_t &flags) {
    const int Ls = t.L - 1;
    for (int c = threadIdx.x; c < t.C; c += blockDim.x) {
        int32_t size = __ldg(t.sizes + c);
        if (size < 2 || size > t.L) {
            flags |= kFlagTable;
            size = size < 2 ? 2 : t.L;
        }
        s_ch[c] = make_int2(__ldg(t.offs + c), size - 2);
    }
    __syncthreads();
    const int total = t.C * Ls;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
        int c = e / Ls, v = e - c * Ls;
        int maxv = s_ch[c].y;
        uint32_t ent = 0u;
        if (v <= maxv) {
            const int32_t *row = t.cdfs + (int64_t)c * t.L;
            int32_t a = __ldg(row + v), b = __ldg(row + v + 1);
            ent = pack_entry(a, b, flags);
            if (s_lut) {
                // buckets whose first slot lies in this symbol's range; the
                // first symbol also owns slots below cdf[0] and the last one
                // the slots above cdf[size-1] (binary-search semantics)
                int lo = v == 0 ? 0 : (int)(ent & 0xFFFFu);
                int hi = v == maxv ? 65536 : (int)(ent & 0xFFFFu) + (int)(ent >> 16) + 1;
                int u0 = (lo + (1 << kLutShift) - 1) >> kLutShift;
                int u1 = (hi + (1 << kLutShift) - 1) >> kLutShift;
                if (u1 > kLutBuckets) u1 = kLutBuckets;
                for (int u = u0; u < u1; ++u) s_lut[c * kLutBuckets + u] = (uint16_t)v;
            }
        }
        s_tab[e] = ent;
    }
    __syncthreads();
}

// Validation of all rows when they are read from global memory.
__device__ void validate_tables_global(const TableArgs &t, uint32_t &flags) {
    for (int c = threadIdx.x; c < t.C; c += blockDim.x) {
        int32_t size = __ldg(t.sizes + c);
        if (size < 2 || size > t.L) {
            flags |= kFlagTable;
            continue;
        }
        const int32_t *row = t.cdfs + (int64_t)c * t.L;
        for (int v = 0; v + 1 < size; ++v) pack_entry(__ldg(row + v), __ldg(row + v + 1), flags);
    }
}

// Full-table accessor (every row of the batch, in shared memory when it
// fits, else read from global memory).  The division magic comes from the
// per-device table g_magic.
template <bool kSmem>
struct Tables {
    const uint32_t *s_tab;
    const int2 *s_ch;
    const uint16_t *s_lut;
    TableArgs g;
    const float *med;  // latent medians (global)

    __device__ __forceinline__ int2 chan(int c) const {
        if (kSmem) return s_ch[c];
        int32_t size = __ldg(g.sizes + c);
        size = size < 2 ? 2 : (size > g.L ? g.L : size);
        return make_int2(__ldg(g.offs + c), size - 2);
    }
    __device__ __forceinline__ uint32_t entry(int c, int v, uint32_t &flags) const {
        if (kSmem) return s_tab[c * (g.L - 1) + v];
        const int32_t *row = g.cdfs + (int64_t)c * g.L;
        return pack_entry(__ldg(row + v), __ldg(row + v + 1), flags);
    }
    __device__ __forceinline__ uint64_t magic(int, int, uint32_t freq) const { return g_magic[freq]; }
    __device__ __forceinline__ float median(int c) const { return __ldg(med + c); }
    // First s in [0, maxv] with cdf[s+1] > slot (maxv if none); returns the
    // symbol and its entry.
    __device__ __forceinline__ int search(int c, int maxv, uint32_t slot, uint32_t &ent, uint32_t &flags) const {
        if (kSmem) {
            int s = s_lut[c * kLutBuckets + (slot >> kLutShift)];
            if (s > maxv) s = maxv;
            const uint32_t *row = s_tab + c * (g.L - 1);
            uint32_t e = row[s];
            while (s < maxv && (e & 0xFFFFu) + (e >> 16) + 1u <= slot) e = row[++s];
            ent = e;
            return s;
        }
        const int32_t *row = g.cdfs + (int64_t)c * g.L;
        int lo = 0, hi = maxv;
        while (lo < hi) {
            int mid = (lo + hi) >> 1;
            if ((uint32_t)__ldg(row + mid + 1) > slot) hi = mid;
            else lo = mid + 1;
        }
        ent = pack_entry(__ldg(row + lo), __ldg(row + lo + 1), flags);
        return lo;
    }
};

// ---------------------------------------------------------------------------
// rANS primitives (rans64_gpu.cuh:21-55, rans64_gpu_v2.cuh:90-120 semantics)
// ---------------------------------------------------------------------------

struct LaneWriter {
    uint32_t *rows;  // stage of this chunk, row j of this lane at j * 32
    int cap;         // rows available
    int j;           // words emitted so far
    __device__ __forceinline__ void emit(uint32_t w) {
        if (j < cap) rows[j * kLanes] = w;
        ++j;
    }
};

__device__ __forceinline__ void put_symbol(uint64_t &x, uint32_t start, uint32_t freq, uint64_t magic,
                                           LaneWriter &w) {
    if (x >= ((uint64_t)freq << 47)) {  // ((L >> 16) << 32) * freq
        w.emit((uint32_t)x);
        x >>= 32;
    }
    // magic = floor((2^64 - 1) / freq), freq in [1, 65536]: q is floor(x / freq)
    // or one less (x < 2^63 after renormalisation), fixed by one correction.
    // freq = 1 gives q = x - 1, corrected to x, r = 0.
    uint64_t q = __umul64hi(x, magic);
    uint64_t rr = x - q * (uint64_t)freq;
    if (rr >= freq) {
        ++q;
        rr -= freq;
    }
    x = (q << 16) + (uint64_t)((uint32_t)rr + start);
}

__device__ __forceinline__ void put_nibble(uint64_t &x, uint32_t val, LaneWriter &w) {
    if (x >= (4096ull << 47)) {  // freq = 1 << (16 - 4)
        w.emit((uint32_t)x);
        x >>= 32;
    }
    x = (x << kBypassBits) | (uint64_t)val;
}

// Escape code of an out-of-range value (warp_ans_kernel_v2.cu:148-164).
__device__ __forceinline__ void put_escape_inl(uint64_t &x, uint32_t raw, LaneWriter &w) {
    int n_bypass = raw ? (31 - __clz(raw)) / (int)kBypassBits + 1 : 0;
    for (int j = n_bypass - 1; j >= 0; --j) put_nibble(x, (raw >> (j * kBypassBits)) & kBypassMax, w);
    int rem = n_bypass, n_full = 0;
    while (rem >= (int)kBypassMax) {
        rem -= (int)kBypassMax;
        ++n_full;
    }
    put_nibble(x, (uint32_t)rem, w);
    for (int k = 0; k < n_full; ++k) put_nibble(x, kBypassMax, w);
}

// Out-of-line escape (rare path): state in and out by value, so the hot
// loop keeps x and the writer in registers and stays small.
struct EscOut {
    uint64_t x;
    int j;
};
__device__ __noinline__ EscOut put_escape_call(uint64_t x, uint32_t raw, uint32_t *rows, int cap, int j) {
    LaneWriter w{rows, cap, j};
    put_escape_inl(x, raw, w);
    return EscOut{x, w.j};
}
__device__ __forceinline__ void put_escape(uint64_t &x, uint32_t raw, LaneWriter &w) {
    const EscOut r = put_escape_call(x, raw, w.rows, w.cap, w.j);
    x = r.x;
    w.j = r.j;
}

// ---------------------------------------------------------------------------
// Block-wide exclusive scan (used by the single "last" CTA)
// ---------------------------------------------------------------------------

__device__ uint64_t block_exclusive_scan(uint64_t v, uint64_t *s_warp, uint64_t &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint64_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint64_t w = lane < nwarps ? s_warp[lane] : 0ull;
        uint64_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint64_t n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        if (lane < nwarps) s_warp[lane] = wi - w;
        if (lane == 31) s_warp[32] = wi;
    }
    __syncthreads();
    uint64_t r = s_warp[warp] + inc - v;
    total = s_warp[32];
    __syncthreads();
    return r;
}

// offsets[c] = sum_{c' < c} rounds[c'] * 32; returns the total (all threads).
__device__ uint64_t scan_rounds(const int32_t *rounds, int64_t n, unsigned long long *offsets, uint64_t *s_warp) {
    const int64_t per = (n + blockDim.x - 1) / blockDim.x;
    const int64_t lo = (int64_t)threadIdx.x * per;
    const int64_t hi = lo + per < n ? lo + per : n;
    uint64_t sum = 0;
    for (int64_t c = lo; c < hi; ++c) sum += (uint64_t)(uint32_t)__ldcg(rounds + c) * kLanes;
    uint64_t total;
    uint64_t run = block_exclusive_scan(sum, s_warp, total);
    for (int64_t c = lo; c < hi; ++c) {
        offsets[c] = run;
        run += (uint64_t)(uint32_t)__ldcg(rounds + c) * kLanes;
    }
    return total;
}

// ---------------------------------------------------------------------------
// Encode
// ---------------------------------------------------------------------------

// Where encode reads its symbols / decode writes its result.
enum Mode : int {
    kModeIdx = 0,      // int32 symbols with explicit indexes[B,N]
    kModeChannel = 1,  // int32 symbols, channel layout index = i / HW
    kModeLatent = 2,   // fp32 latent y with per-channel medians, channel layout:
                       // symbol = (int)rint(y - median)  (factorized.py:46-49),
                       // y_hat = (float)symbol + median  (factorized.py:99-101)
};

struct EncParams {
    const int32_t *__restrict__ sym;
    const int32_t *__restrict__ idx;     // kModeIdx only
    const float *__restrict__ y;         // kModeLatent only
    const float *__restrict__ medians;   // kModeLatent only
    TableArgs t;
    int B, N, P, K, chunk_len, HW;
    int rows_cap;
    int64_t chunks;
    Control *ctrl;
    int32_t *rounds;
    int32_t *used;
    unsigned long long *offsets;
    uint32_t *stage;
    uint32_t *max_rounds_out;
    long long *status_out;  // optional: a mapped host slot that also receives the 8 status words
};

constexpr int kPrefetch = 16;  // symbols each lane loads ahead of the coding chain
constexpr int kBatch = 8;      // symbols whose table lookups are issued together

// Loads lane symbols t0 .. t0+7 (reverse order: position last - 32 t) of one
// image row, with their indexes in kModeIdx; latent values as float bits.
template <int kMode>
__device__ __forceinline__ void load_batch(const EncParams &p, int64_t row0, int last, int t0, int n,
                                           int32_t (&v)[kPrefetch], int32_t (&iv)[kPrefetch]) {
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
        const int t = t0 + u;
        v[u] = 0;
        iv[u] = 0;
        if (t < n) {
            const int64_t pos = row0 + last - t * kLanes;
            v[u] = kMode == kModeLatent ? __float_as_int(__ldg(p.y + pos)) : __ldg(p.sym + pos);
            if (kMode == kModeIdx) iv[u] = __ldg(p.idx + pos);
        }
    }
}

// Codes one chunk: each lane runs its symbols last to first (prefetching the
// next kPrefetch symbols while coding the current ones), staging its words
// in emission order, then the warp records used words and max_rounds.
template <int kMode, class Tab>
__device__ __forceinline__ void encode_chunk(const EncParams &p, const Tab &tab, int64_t chunk, int lane,
                                             uint32_t &flags, unsigned int &my_max_used) {
    constexpr bool kIdx = kMode == kModeIdx;
    const int C = p.t.C;
    const int b = (int)(chunk / p.K);
    const int k = (int)(chunk - (int64_t)b * p.K);
    const int start = k * p.chunk_len;
    const int end = min(start + p.chunk_len, p.N);
    const int first = start + lane;
    LaneWriter w{p.stage + chunk * (int64_t)p.rows_cap * kLanes + lane, p.rows_cap, 0};
    if (first < end) {
        const int n = (end - 1 - first) / kLanes + 1;
        const int last = first + (n - 1) * kLanes;
        int ct = last / p.HW, rem = last - ct * p.HW;  // channel-layout position tracker
        const int64_t row0 = (int64_t)b * p.N;
        uint64_t x = kRansL;
        int32_t cur[kPrefetch], icur[kPrefetch];
        load_batch<kMode>(p, row0, last, 0, n, cur, icur);
        for (int t0 = 0; t0 < n; t0 += kPrefetch) {
            // the next batch's loads are in flight while this one is coded
            int32_t nxt[kPrefetch], inxt[kPrefetch];
            load_batch<kMode>(p, row0, last, t0 + kPrefetch, n, nxt, inxt);
#pragma unroll
            for (int h = 0; h < kPrefetch; h += kBatch) {
                // Phase A: everything that does not depend on the coder
                // state, for kBatch symbols (their shared-memory reads are
                // independent and overlap).
                uint32_t ent[kBatch], raw[kBatch];
                uint64_t mag[kBatch];
                uint32_t esc = 0u;
                const int nrem = n - (t0 + h);  // symbols left from this batch on (may be <= 0)
                const int nb = min(kBatch, nrem);
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    int32_t s;
                    if (kMode == kModeLatent) {
                        // torch.round (half to even) then .int(), both in fp32
                        s = __float2int_rz(rintf(__int_as_float(cur[h + u]) - tab.median(ct)));
                    } else {
                        s = cur[h + u];
                    }
                    int c = ct;
                    if (kIdx) {
                        const int32_t ci = icur[h + u];
                        if (u < nb) {
                            if (ci != ct) flags |= kFlagNonChannel;
                            if ((unsigned)ci >= (unsigned)C) flags |= kFlagIndexRange;
                        }
                        c = (unsigned)ci < (unsigned)C ? ci : 0;
                    }
                    const int2 ch = tab.chan(c);
                    int32_t value = (int32_t)((uint32_t)s - (uint32_t)ch.x);
                    const int32_t maxv = ch.y;
                    // negative: raw = -2v - 1; at/above max: raw = 2(v - max)
                    raw[u] = value < 0 ? 0u - 2u * (uint32_t)value - 1u : ((uint32_t)value - (uint32_t)maxv) * 2u;
                    const bool out_of_range = value < 0 || value >= maxv;
                    if (out_of_range && u < nb) esc |= 1u << u;
                    value = out_of_range ? maxv : value;
                    uint32_t tf = 0u;
                    ent[u] = tab.entry(c, value, u < nb ? flags : tf);
                    mag[u] = tab.magic(c, value, (ent[u] >> 16) + 1u);
                    // step to the next symbol's channel only when one follows,
                    // so that ct always names a row this chunk stages
                    if (u + 1 < nrem) {
                        rem -= kLanes;
                        while (rem < 0) {
                            rem += p.HW;
                            --ct;
                        }
                    }
                }
                // Phase B: the coder chain.
                if (nb >= kBatch && esc == 0u) {
#pragma unroll
                    for (int u = 0; u < kBatch; ++u)
                        put_symbol(x, ent[u] & 0xFFFFu, (ent[u] >> 16) + 1u, mag[u], w);
                } else {
#pragma unroll
                    for (int u = 0; u < kBatch; ++u) {
                        if (u < nb) {
                            if ((esc >> u) & 1u) put_escape(x, raw[u], w);
                            put_symbol(x, ent[u] & 0xFFFFu, (ent[u] >> 16) + 1u, mag[u], w);
                        }
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kPrefetch; ++u) {
                cur[u] = nxt[u];
                icur[u] = inxt[u];
            }
        }
        w.emit((uint32_t)(x >> 32));  // flush: decode order is low, high, ...
        w.emit((uint32_t)x);
    }
    const int used = w.j;
    int rounds = used;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rounds = max(rounds, __shfl_xor_sync(0xffffffffu, rounds, o));
    p.used[chunk * kLanes + lane] = used;
    if (lane == 0) {
        p.rounds[chunk] = rounds;
        p.max_rounds_out[chunk] = (uint32_t)rounds;
    }
    if ((unsigned)rounds > my_max_used) my_max_used = (unsigned)rounds;
}

// CTA summary; the last CTA to finish computes the chunk offsets and the
// status block the host reads, and re-arms the control block.
__device__ __forceinline__ void finish_encode(const EncParams &p, uint32_t flags, unsigned int my_max_used) {
    __shared__ uint64_t s_warp[33];
    __shared__ unsigned int s_flags, s_max_used;
    __shared__ int s_last;
    if (my_max_used > (unsigned)p.rows_cap) flags |= kFlagOverflow;
    __syncthreads();
    if (threadIdx.x == 0) {
        s_flags = 0;
        s_max_used = 0;
    }
    __syncthreads();
    if (flags) atomicOr(&s_flags, flags);
    if (my_max_used) atomicMax(&s_max_used, my_max_used);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (s_flags) atomicOr(&p.ctrl->flags, s_flags);
        atomicMax(&p.ctrl->max_used, s_max_used);
        __threadfence();
        s_last = atomicAdd(&p.ctrl->done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    uint64_t total = scan_rounds(p.rounds, p.chunks, p.offsets, s_warp);
    if (threadIdx.x == 0) {
        volatile Control *ctl = p.ctrl;
        ctl->status[kStTotalWords] = (long long)total;
        ctl->status[kStFlags] = (long long)ctl->flags;
        ctl->status[kStMaxUsed] = (long long)ctl->max_used;
        ctl->status[kStRowsCap] = p.rows_cap;
        ctl->flags = 0;
        ctl->max_used = 0;
        ctl->done = 0;
        // the host's copy, visible to it once the kernel has completed
        if (p.status_out)
            for (int i = 0; i < 8; ++i) p.status_out[i] = ctl->status[i];
    }
}

// Explicit indexes: any row can be used by any symbol, so every CTA stages
// all rows once and its warps take chunks in a grid-stride loop.
template <bool kSmem>
__global__ void __launch_bounds__(kThreads) encode_kernel(EncParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t flags = 0;
    const int C = p.t.C;
    uint32_t *s_tab = reinterpret_cast<uint32_t *>(smem);
    int2 *s_ch = reinterpret_cast<int2 *>(smem + (((int64_t)C * (p.t.L - 1) * 4 + 15) & ~15ll));
    if (kSmem) {
        stage_tables(p.t, s_tab, s_ch, nullptr, flags);
    } else {
        if (blockIdx.x == 0) validate_tables_global(p.t, flags);
        __syncthreads();
    }
    Tables<kSmem> tab{s_tab, s_ch, nullptr, p.t, p.medians};
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t warp_stride = (int64_t)gridDim.x * warps;
    unsigned int my_max_used = 0;
    for (int64_t chunk = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); chunk < p.chunks; chunk += warp_stride)
        encode_chunk<kModeIdx>(p, tab, chunk, lane, flags, my_max_used);
    finish_encode(p, flags, my_max_used);
}

// Channel-layout indexes with the CDF rows read from global memory: the
// fallback of encode_lanes_kernel when a chunk group's rows do not fit in
// shared memory.  A CTA of W warps takes groups (k, images b0 .. b0+W-1).
template <int kMode>
__global__ void __launch_bounds__(kThreads) encode_group_kernel(EncParams p) {
    uint32_t flags = 0;
    unsigned int my_max_used = 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int nbb = (p.B + W - 1) / W;
    const int64_t groups = (int64_t)p.K * nbb;
    Tables<false> tg{nullptr, nullptr, nullptr, p.t, p.medians};
    if (blockIdx.x == 0) validate_tables_global(p.t, flags);
    for (int64_t g = blockIdx.x; g < groups; g += gridDim.x) {
        const int k = (int)(g % p.K), bb = (int)(g / p.K);
        const int b = bb * W + warp;
        if (b < p.B) encode_chunk<kMode>(p, tg, (int64_t)b * p.K + k, lane, flags, my_max_used);
    }
    finish_encode(p, flags, my_max_used);
}

struct PackParams {
    const Control *ctrl;
    const int32_t *rounds;
    const int32_t *used;
    const unsigned long long *offsets;
    const uint32_t *stage;
    int64_t chunks;
    int B, N, K, chunk_len;
    int64_t header_bytes;
    int64_t packed_bytes;
    uint8_t *packed;
};

// ---------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------

struct DecPrepParams {
    const uint8_t *packed;
    const uint32_t *max_rounds;
    int64_t chunks;
    int B, N, K, chunk_len;
    int64_t header_bytes, packed_bytes;
    Control *ctrl;
    unsigned long long *offsets;
};

// Header check (coders/warp_div.py:161-176), rounds >= 2 and total length
// (coders/warp_div.py:62-67), and chunk offsets.
__global__ void __launch_bounds__(1024) decode_prep_kernel(DecPrepParams p) {
    __shared__ uint64_t s_warp[33];
    __shared__ unsigned int s_flags;
    if (threadIdx.x == 0) s_flags = 0;
    __syncthreads();
    uint32_t flags = 0;
    const uint32_t *hdr = reinterpret_cast<const uint32_t *>(p.packed);
    if (threadIdx.x == 0) {
        if (hdr[0] != (uint32_t)p.N || hdr[1] != (uint32_t)p.chunk_len ||
            hdr[2] != (((uint32_t)p.B << 16) | (uint32_t)p.K) || hdr[3] != ((32u << 16) | 2u) || hdr[4] != 0u ||
            hdr[5] != 0u)
            flags |= kFlagHeader;
    }
    // round table: max_rounds as int32 at word 8 (fits: header_bytes >= 32 + 4*B*K)
    const int32_t *mr = reinterpret_cast<const int32_t *>(p.max_rounds);
    for (int64_t c = threadIdx.x; c < p.chunks; c += blockDim.x) {
        if ((int32_t)hdr[8 + c] != mr[c]) flags |= kFlagRounds;
        if (p.max_rounds[c] < 2u || p.max_rounds[c] > 0x7fffffffu) flags |= kFlagCorrupt;
    }
    uint64_t total = scan_rounds(mr, p.chunks, p.offsets, s_warp);
    if (threadIdx.x == 0 && p.header_bytes + 4 * (int64_t)total != p.packed_bytes) flags |= kFlagCorrupt;
    if (flags) atomicOr(&s_flags, flags);
    __syncthreads();
    if (threadIdx.x == 0 && s_flags) atomicOr(&p.ctrl->flags, s_flags);
}

struct DecParams {
    const uint8_t *__restrict__ packed;
    int64_t header_bytes;
    const uint32_t *__restrict__ max_rounds;
    const int32_t *__restrict__ idx;       // kModeIdx only
    const float *__restrict__ medians;     // kModeLatent only
    float *__restrict__ y_out;             // kModeLatent only
    TableArgs t;
    int B, N, K, chunk_len, HW;
    int64_t chunks;
    Control *ctrl;
    const unsigned long long *offsets;
    int32_t *__restrict__ out;
    int group_warps;  // lanes decode: warps that decode (one image each); the CTA's others only stage
};

// The lane's words in decode order, read four at a time: r0..r3 hold words
// 4m .. 4m+3 (loaded), f0..f3 words 4m+4 .. 4m+7 (in flight).  Consuming the
// last ready word moves the in-flight quad in and issues the next one, so a
// register move only ever waits on loads issued four refills earlier.
struct LaneReader {
    const uint32_t *__restrict__ base;  // chunk body + lane
    int word, rounds;                   // index of the next word
    bool bad;
    uint32_t r0, r1, r2, r3, f0, f1, f2, f3;
    __device__ __forceinline__ uint32_t fetch(int j) const {
        return j < rounds ? __ldg(base + (int64_t)j * kLanes) : 0u;
    }
    __device__ __forceinline__ void start() {
        r0 = fetch(0);
        r1 = fetch(1);
        r2 = fetch(2);
        r3 = fetch(3);
        f0 = fetch(4);
        f1 = fetch(5);
        f2 = fetch(6);
        f3 = fetch(7);
    }
    __device__ __forceinline__ uint32_t next() {
        if (word >= rounds) bad = true;
        const int k = word & 3;
        const uint32_t v = k == 0 ? r0 : k == 1 ? r1 : k == 2 ? r2 : r3;
        ++word;
        if (k == 3) {
            r0 = f0;
            r1 = f1;
            r2 = f2;
            r3 = f3;
            f0 = fetch(word + 4);
            f1 = fetch(word + 5);
            f2 = fetch(word + 6);
            f3 = fetch(word + 7);
        }
        return v;
    }
};

__device__ __forceinline__ uint32_t get_nibble(uint64_t &x, LaneReader &rd) {
    uint32_t v = (uint32_t)x & kBypassMax;
    x >>= kBypassBits;
    if (x < kRansL) x = (x << 32) | (uint64_t)rd.next();
    return v;
}

// Escape decode (warp_ans_kernel.cu:308-325).  Returns false on a corrupt
// count (the format never needs more than 8 nibbles).
__device__ __forceinline__ bool get_escape_inl(uint64_t &x, LaneReader &rd, int32_t maxv, int32_t &value) {
    uint32_t v = get_nibble(x, rd);
    uint32_t n_bypass = v;
    while (v == kBypassMax && !rd.bad) {
        v = get_nibble(x, rd);
        n_bypass += v;
    }
    if (n_bypass > 8u || rd.bad) return false;
    uint32_t raw = 0;
    for (uint32_t j = 0; j < n_bypass; ++j) raw |= get_nibble(x, rd) << (j * kBypassBits);
    int32_t val = (int32_t)raw >> 1;  // int32 arithmetic shift, as in the reference
    if (raw & 1u) val = -val - 1;
    else val = (int32_t)((uint32_t)val + (uint32_t)maxv);
    value = val;
    return true;
}

struct EscIn {
    uint64_t x;
    LaneReader rd;
    int32_t value;
    bool ok;
};
__device__ __noinline__ EscIn get_escape_call(uint64_t x, LaneReader rd, int32_t maxv) {
    EscIn r;
    r.ok = get_escape_inl(x, rd, maxv, r.value);
    r.x = x;
    r.rd = rd;
    return r;
}
__device__ __forceinline__ bool get_escape(uint64_t &x, LaneReader &rd, int32_t maxv, int32_t &value) {
    const EscIn r = get_escape_call(x, rd, maxv);
    x = r.x;
    rd = r.rd;
    value = r.value;
    return r.ok;
}

// Decodes one chunk: each lane reads its state, then its symbols first to
// last, refilling from a look-ahead queue of its payload words.
template <int kMode, class Tab>
__device__ __forceinline__ void decode_chunk(const DecParams &p, const Tab &tab, int64_t chunk, int lane,
                                             uint32_t &flags) {
    constexpr bool kIdx = kMode == kModeIdx;
    const int C = p.t.C;
    const uint32_t *body = reinterpret_cast<const uint32_t *>(p.packed + p.header_bytes);
    const int b = (int)(chunk / p.K);
    const int k = (int)(chunk - (int64_t)b * p.K);
    const int64_t start64 = (int64_t)k * p.chunk_len;
    if (start64 >= p.N) return;
    const int start = (int)start64;
    const int end = (int)min(start64 + p.chunk_len, (int64_t)p.N);
    // the chunk's word offset: from the prep kernel's scan, or (payloads
    // the host has validated, few chunks) summed here by the whole warp over
    // the rounds of the chunks before it
    uint64_t off;
    if (p.offsets) {
        off = p.offsets[chunk];
    } else {
        uint64_t sum = 0;
        for (int64_t c = lane; c < chunk; c += kLanes) sum += (uint64_t)__ldg(p.max_rounds + c);
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        off = sum * kLanes;
    }
    const int first = start + lane;
    if (first >= end) return;
    LaneReader rd{body + off + lane, 0, (int)p.max_rounds[chunk], false, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    rd.start();
    uint64_t x = (uint64_t)rd.next();
    x |= (uint64_t)rd.next() << 32;
    const int32_t *irow = kIdx ? p.idx + (int64_t)b * p.N : nullptr;
    int32_t *orow = kMode == kModeLatent ? nullptr : p.out + (int64_t)b * p.N;
    float *yrow = kMode == kModeLatent ? p.y_out + (int64_t)b * p.N : nullptr;
    int ct = first / p.HW, rem = first - ct * p.HW;
    const int n = (end - 1 - first) / kLanes + 1;
    int32_t icur[kPrefetch], inxt[kPrefetch];
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) icur[u] = (kIdx && u < n) ? __ldg(irow + first + u * kLanes) : 0;
    for (int t0 = 0; t0 < n && !rd.bad; t0 += kPrefetch) {
#pragma unroll
        for (int u = 0; u < kPrefetch; ++u)  // next batch of indexes in flight
            inxt[u] = (kIdx && t0 + kPrefetch + u < n) ? __ldg(irow + first + (t0 + kPrefetch + u) * kLanes) : 0;
#pragma unroll
        for (int u = 0; u < kPrefetch; ++u) {
            if (t0 + u < n && !rd.bad) {
                const int i = first + (t0 + u) * kLanes;
                int c = ct;
                if (kIdx) {
                    const int32_t ci = icur[u];
                    if (ci != ct) flags |= kFlagNonChannel;
                    if ((unsigned)ci >= (unsigned)C) {
                        flags |= kFlagIndexRange;
                        c = 0;
                    } else {
                        c = ci;
                    }
                }
                const int2 ch = tab.chan(c);
                const uint32_t slot = (uint32_t)x & 0xFFFFu;
                uint32_t e;
                int32_t value = tab.search(c, ch.y, slot, e, flags);
                x = (uint64_t)((e >> 16) + 1u) * (x >> 16) + (uint64_t)slot - (uint64_t)(e & 0xFFFFu);
                if (x < kRansL) x = (x << 32) | (uint64_t)rd.next();
                if (value == ch.y && !get_escape(x, rd, ch.y, value)) rd.bad = true;
                if (!rd.bad) {
                    const int32_t sym = (int32_t)((uint32_t)value + (uint32_t)ch.x);
                    if (kMode == kModeLatent) yrow[i] = __int2float_rn(sym) + tab.median(c);
                    else orow[i] = sym;
                }
                rem += kLanes;
                while (rem >= p.HW) {
                    rem -= p.HW;
                    ++ct;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kPrefetch; ++u) icur[u] = inxt[u];
    }
    if (rd.bad) flags |= kFlagCorrupt;
}

__device__ __forceinline__ void finish_decode(const DecParams &p, uint32_t flags) {
    __shared__ unsigned int s_flags;
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) s_flags = 0;
    __syncthreads();
    if (flags) atomicOr(&s_flags, flags);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (s_flags) atomicOr(&p.ctrl->flags, s_flags);
        __threadfence();
        s_last = atomicAdd(&p.ctrl->done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
        __threadfence();
        volatile Control *ctl = p.ctrl;
        ctl->status[kStFlags] = (long long)ctl->flags;
        ctl->flags = 0;
        ctl->done = 0;
    }
}

// prep (or an earlier CTA) found a bad payload or table: decode nothing
__device__ __forceinline__ bool decode_skip(const DecParams &p) {
    return (*((volatile unsigned int *)&p.ctrl->flags) & ~kFlagNonChannel) != 0;
}

// All rows staged per CTA (explicit indexes, or a chunk_len that is not a
// whole number of channels), grid-stride over chunks.
template <int kMode, bool kSmem>
__global__ void __launch_bounds__(kThreads) decode_kernel(DecParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t flags = 0;
    const bool skip = decode_skip(p);
    const int C = p.t.C;
    const int64_t tab_bytes = ((int64_t)C * (p.t.L - 1) * 4 + 15) & ~15ll;
    uint32_t *s_tab = reinterpret_cast<uint32_t *>(smem);
    int2 *s_ch = reinterpret_cast<int2 *>(smem + tab_bytes);
    uint16_t *s_lut = reinterpret_cast<uint16_t *>(smem + tab_bytes + (int64_t)C * 8);
    if (kSmem) {
        stage_tables(p.t, s_tab, s_ch, s_lut, flags);
    } else {
        if (blockIdx.x == 0) validate_tables_global(p.t, flags);
        __syncthreads();
    }
    Tables<kSmem> tab{s_tab, s_ch, s_lut, p.t, p.medians};
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t warp_stride = (int64_t)gridDim.x * warps;
    for (int64_t chunk = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); !skip && chunk < p.chunks;
         chunk += warp_stride)
        decode_chunk<kMode>(p, tab, chunk, lane, flags);
    finish_decode(p, flags);
}

// Channel-layout indexes with the CDF rows read from global memory: the
// fallback of decode_lanes_kernel when a group's rows do not fit in shared
// memory.
template <int kMode>
__global__ void __launch_bounds__(kThreads) decode_group_kernel(DecParams p) {
    __shared__ int s_skip;
    uint32_t flags = 0;
    if (threadIdx.x == 0) s_skip = decode_skip(p) ? 1 : 0;
    __syncthreads();
    const bool skip = s_skip != 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int nbb = (p.B + W - 1) / W;
    const int64_t groups = (int64_t)p.K * nbb;
    Tables<false> tg{nullptr, nullptr, nullptr, p.t, p.medians};
    if (blockIdx.x == 0) validate_tables_global(p.t, flags);
    for (int64_t g = blockIdx.x; g < groups && !skip; g += gridDim.x) {
        const int k = (int)(g % p.K), bb = (int)(g / p.K);
        const int b = bb * W + warp;
        if (b < p.B) decode_chunk<kMode>(p, tg, (int64_t)b * p.K + k, lane, flags);
    }
    finish_decode(p, flags);
}

// ---------------------------------------------------------------------------
// Chunk-group coder with per-symbol chains free of divergent branches
// ---------------------------------------------------------------------------
// The group kernels above resolve each symbol with table searches and a
// look-ahead word queue whose refills branch per lane, so a warp executes
// both sides of every renormalisation and search.  These kernels keep the
// same decomposition (a CTA stages one chunk group's P rows, each warp codes
// one chunk) and the same arithmetic, but every step of a symbol is a fixed
// instruction sequence:
//  * encode reads one 16-byte entry {magic lo, magic hi, freq, start} per
//    symbol; the renormalisation word is a predicated store; the quotient
//    estimate floor(x * magic / 2^64) is q or q - 1 and the remainder fits
//    in 32 bits, so the correction is one compare on 32-bit values;
//  * decode reads one 8-byte bucket entry {entry of the bucket's first
//    symbol, first | last symbol of the bucket} per symbol: a bucket that
//    holds one symbol (nearly every lookup) needs no search.  The refill
//    word is a candidate loaded one symbol ahead, so the refill itself is a
//    predicated register move; rows of the lane's stream are prefetched into
//    L1 a few words ahead.
// Channel-dependent values (row pointers, offset, escape symbol, median)
// change only when a lane crosses into the next channel.

// Shared-memory layout of one group's rows for the lanes kernels.
struct LanesSmem {
    int64_t ent, chan, lut, bytes;
    int lut_shift;  // decode: bucket = slot >> lut_shift
};

// Decode buckets per row: the largest power of two in [32, 2048] with
// P * buckets <= 8192 (64 KB of 8-byte entries).
__host__ __device__ inline int lanes_lut_shift(int P) {
    int shift = 5;
    while (shift < 11 && (int64_t)(65536 >> shift) * P > 8192) ++shift;
    return shift;
}

__host__ __device__ inline LanesSmem lanes_smem(int P, int L, bool encode) {
    const int64_t ents = (int64_t)P * (L - 1);
    LanesSmem s;
    s.ent = 0;
    s.chan = (ents * (encode ? 16 : 4) + 15) & ~15ll;
    s.lut = s.chan + (int64_t)P * 16;
    s.lut_shift = lanes_lut_shift(P);
    s.bytes = s.lut + (encode ? 0 : (int64_t)P * (65536 >> s.lut_shift) * 8);
    return s;
}

// First symbol s in [0, maxv] whose range reaches slot (end(s) - 1 >= slot),
// maxv if none: the reference's warp_cdf_find_symbol (warp_ans_kernel.cu:
// 28-39) over decode entries start | (end - 1) << 16.
__device__ __forceinline__ int lanes_find(const uint32_t *row, int lo, int hi, uint32_t slot) {
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((row[mid] >> 16) >= slot) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// Stages rows [c0, c0 + nc): channel info {median bits, offset, maxv}, the
// per-symbol entries and (decode) the slot buckets.  Ends with a barrier.
//
// Decode bucket u of a row covers slots [u << shift, (u + 1) << shift).  Its
// 8-byte entry holds the decode entry of s0, the symbol of the bucket's
// first slot (the first symbol also owns the slots below cdf[0], the last
// one those above cdf[size - 1]), and in its high word either
//  * kPair: end(s0 + 1) - 1 | s0 << 16, so that a slot past s0's range
//    resolves to s0 + 1 without another read; a slot past that one too (a
//    bucket of three or more symbols) is searched in [s0 + 2, maxv];
//  * otherwise: s0 | s1 << 16, s1 the symbol of the bucket's last slot, so
//    that a slot past s0's range is searched in (s0, s1].
// Each thread fills a run of consecutive buckets of one row, walking the
// row's symbols forward, so a row costs its buckets plus its symbols.
template <bool kPair>
__device__ void stage_lanes(const TableArgs &t, int c0, int nc, bool encode, unsigned char *smem,
                            const LanesSmem &ls, const float *medians, uint32_t &flags) {
    const int Ls = t.L - 1;
    int4 *chan = reinterpret_cast<int4 *>(smem + ls.chan);
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        int32_t size = __ldg(t.sizes + c0 + c);
        if (size < 2 || size > t.L) {
            flags |= kFlagTable;
            size = size < 2 ? 2 : t.L;
        }
        chan[c] = make_int4(medians ? __float_as_int(__ldg(medians + c0 + c)) : 0, __ldg(t.offs + c0 + c), size - 2, 0);
    }
    __syncthreads();
    const int total = nc * Ls;
#pragma unroll 4
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
        const int c = e / Ls, v = e - c * Ls;
        uint32_t start = 0u, freq = 1u;
        if (v <= chan[c].z) {
            const int32_t *row = t.cdfs + (int64_t)(c0 + c) * t.L;
            const uint32_t ent = pack_entry(__ldg(row + v), __ldg(row + v + 1), flags);
            start = ent & 0xFFFFu;
            freq = (ent >> 16) + 1u;
        }
        if (encode) {
            const uint64_t m = (~0ull) / (uint64_t)freq;
            reinterpret_cast<uint4 *>(smem + ls.ent)[e] = make_uint4((uint32_t)m, (uint32_t)(m >> 32), freq, start);
        } else {
            reinterpret_cast<uint32_t *>(smem + ls.ent)[e] = start | ((start + freq - 1u) << 16);
        }
    }
    __syncthreads();
    if (encode) return;
    const uint32_t *ent = reinterpret_cast<const uint32_t *>(smem + ls.ent);
    uint2 *lut = reinterpret_cast<uint2 *>(smem + ls.lut);
    // A warp fills a row's buckets (or a slice of them, when the CTA has
    // more warps than rows): lane l takes buckets l, l + 32, ..., so that a
    // warp's stores hit consecutive words, and walks its symbol forward from
    // one of its buckets to the next (a binary search finds the first).
    const int shift = ls.lut_shift, buckets = 65536 >> shift;
    const int warps = (int)(blockDim.x >> 5), wid = (int)(threadIdx.x >> 5), ln = (int)(threadIdx.x & 31);
    int parts = 1;
    while (nc > 0 && 2 * parts * nc <= warps && buckets / (2 * parts) >= 32) parts *= 2;
    const int span = buckets / parts;
    for (int item = wid; item < nc * parts; item += warps) {
        const int c = item / parts, u0 = (item - c * parts) * span;
        const uint32_t *row = ent + c * Ls;
        const int maxv = chan[c].z;
        uint2 *lrow = lut + (int64_t)c * buckets;
        int s = lanes_find(row, 0, maxv, (uint32_t)(u0 + ln) << shift), s1 = s;
        for (int u = u0 + ln; u < u0 + span; u += 32) {
            const uint32_t first = (uint32_t)u << shift, last = first + (1u << shift) - 1u;
            while (s < maxv && (row[s] >> 16) < first) ++s;
            uint32_t hi;
            if (kPair) {
                hi = (s < maxv ? row[s + 1] >> 16 : 0xFFFFu) | ((uint32_t)s << 16);
            } else {
                s1 = max(s1, s);
                while (s1 < maxv && (row[s1] >> 16) < last) ++s1;
                hi = (uint32_t)s | ((uint32_t)s1 << 16);
            }
            lrow[u] = make_uint2(row[s], hi);
        }
    }
    __syncthreads();
}

// One coder step of the encode (Rans64EncPutV2 semantics,
// rans64_gpu_v2.cuh:35-65): the renormalisation word is a predicated store,
// and floor(x * magic / 2^64) is floor(x / freq) or one less (x < 2^63
// after renormalisation), so the remainder is below 2 * freq and its low 32
// bits are exact.  kCheck bounds the staging store by the lane's capacity.
template <bool kCheck>
__device__ __forceinline__ void enc_step(uint64_t &x, int &j, uint32_t *__restrict__ wrow, int cap, const uint4 e) {
    const uint32_t freq = e.z;
    uint32_t xl = (uint32_t)x, xh = (uint32_t)(x >> 32);
    const bool rn = xh >= (freq << 15);  // x >= ((L >> 16) << 32) * freq
    if (rn && (!kCheck || j < cap)) wrow[(int64_t)j * kLanes] = xl;
    j += rn ? 1 : 0;
    xl = rn ? xh : xl;
    xh = rn ? 0u : xh;
    uint64_t q = __umul64hi(((uint64_t)xh << 32) | xl, ((uint64_t)e.y << 32) | e.x);
    uint32_t r = xl - (uint32_t)q * freq;
    const bool c = r >= freq;
    q += c ? 1u : 0u;
    r -= c ? freq : 0u;
    x = (q << 16) + (uint64_t)(r + e.w);
}

// Escape code (bypass nibbles) of an out-of-range value, from the value
// and its channel's escape symbol maxv: negative v gives raw = -2v - 1,
// v >= maxv gives raw = 2(v - maxv) (warp_ans_kernel_v2.cu:148-164).
__device__ __forceinline__ uint32_t escape_raw(int32_t value, int32_t maxv) {
    return value < 0 ? 0u - 2u * (uint32_t)value - 1u : ((uint32_t)value - (uint32_t)maxv) * 2u;
}

// Encodes one chunk: each lane runs its symbols last to first, in batches
// of 8 whose symbols are loaded one batch ahead.  A batch whose symbols lie
// in one channel (every batch when HW is a multiple of 256) takes the fast
// path: its table entries are read before its coder steps, and when no lane
// of the warp escapes and every lane has room for 8 more words the steps
// have no per-symbol checks.  Other batches, the ragged end and escapes go
// through the checked per-symbol path.
//
// With explicit indexes (kModeIdx) each batch also checks, by warp vote,
// that its indexes are the channel layout the group staged; a batch with
// any other index takes the checked path, where a symbol whose row lies
// outside the group reads its entry from global memory (and the call
// reports that the indexes are not the channel layout).
template <int kMode>
__device__ __forceinline__ void encode_lanes(const EncParams &p, const uint4 *__restrict__ ent,
                                             const int4 *__restrict__ chan, int c0, int nc, int Ls, int64_t chunk,
                                             int lane, uint32_t &flags, unsigned int &my_max_used) {
    constexpr int kB = 8, kH = 4;
    constexpr bool kIdx = kMode == kModeIdx;
    const int b = (int)(chunk / p.K);
    const int k = (int)(chunk - (int64_t)b * p.K);
    const int start = k * p.chunk_len;
    const int end = min(start + p.chunk_len, p.N);
    const int first = start + lane;
    uint32_t *const wrow = p.stage + chunk * (int64_t)p.rows_cap * kLanes + lane;
    const int cap = p.rows_cap;
    int j = 0;
    const int n = first < end ? (end - 1 - first) / kLanes + 1 : 0;
    // every lane runs the same number of batches (the warp's longest), so
    // that the warp votes below always see all 32 lanes; a lane past its
    // own symbols takes the guarded path and does nothing
    int nmax = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, o));
    {
        const int last = first + (max(n, 1) - 1) * kLanes;
        int ct = n > 0 ? last / p.HW : c0, rem = n > 0 ? last - ct * p.HW : 0;
        int4 ch = chan[ct - c0];
        const uint4 *row = ent + (ct - c0) * Ls;
        const int64_t pos_last = (int64_t)b * p.N + last;
        const int32_t *src = kMode == kModeLatent ? reinterpret_cast<const int32_t *>(p.y) + pos_last : p.sym + pos_last;
        const int32_t *isrc = kIdx ? p.idx + pos_last : nullptr;
        uint64_t x = kRansL;
        int32_t cur[kB], nxt[kB];
        int32_t icur[kIdx ? kB : 1], inxt[kIdx ? kB : 1];
#pragma unroll
        for (int u = 0; u < kB; ++u) {
            cur[u] = u < n ? __ldg(src - u * kLanes) : 0;
            if (kIdx) icur[u] = u < n ? __ldg(isrc - u * kLanes) : 0;
        }
        for (int t0 = 0; t0 < nmax; t0 += kB) {
            if (t0 + 2 * kB <= n) {
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    nxt[u] = __ldg(src - (t0 + kB + u) * kLanes);
                    if (kIdx) inxt[u] = __ldg(isrc - (t0 + kB + u) * kLanes);
                }
            } else {
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    nxt[u] = t0 + kB + u < n ? __ldg(src - (t0 + kB + u) * kLanes) : 0;
                    if (kIdx) inxt[u] = t0 + kB + u < n ? __ldg(isrc - (t0 + kB + u) * kLanes) : 0;
                }
            }
            // this lane's symbols t0 .. t0 + 7 all lie in channel ct when the
            // position of the 8th is still at or above the channel's start
            bool one_channel = t0 + kB <= n && rem >= (kB - 1) * kLanes;
            if (kIdx) {
#pragma unroll
                for (int u = 0; u < kB; ++u) one_channel = one_channel && icur[u] == ct;
            }
            if (__all_sync(0xffffffffu, one_channel)) {
                const int32_t off = ch.y, maxv = ch.z;
                // two halves of four: a half's entries are read before its
                // coder steps (fewer live registers than a batch of eight)
#pragma unroll
                for (int h = 0; h < kB; h += kH) {
                    uint4 e[kH];
                    int32_t val[kH];
                    uint32_t esc = 0u;
#pragma unroll
                    for (int u = 0; u < kH; ++u) {
                        int32_t s;
                        if (kMode == kModeLatent) s = __float2int_rn(__int_as_float(cur[h + u]) - __int_as_float(ch.x));
                        else s = cur[h + u];
                        val[u] = (int32_t)((uint32_t)s - (uint32_t)off);
                        const bool oor = (uint32_t)val[u] >= (uint32_t)maxv;  // value < 0 or value >= maxv
                        esc |= oor ? 1u << u : 0u;
                        e[u] = row[oor ? maxv : val[u]];
                    }
                    if (__all_sync(0xffffffffu, esc == 0u && j + kH <= cap)) {
#pragma unroll
                        for (int u = 0; u < kH; ++u) enc_step<false>(x, j, wrow, cap, e[u]);
                    } else {
#pragma unroll
                        for (int u = 0; u < kH; ++u) {
                            if (esc & (1u << u)) {
                                const EscOut r = put_escape_call(x, escape_raw(val[u], maxv), wrow, cap, j);
                                x = r.x;
                                j = r.j;
                            }
                            enc_step<true>(x, j, wrow, cap, e[u]);
                        }
                    }
                }
                rem -= kB * kLanes;
                if (rem < 0 && t0 + kB < n) {
                    do {
                        rem += p.HW;
                        --ct;
                    } while (rem < 0);
                    ch = chan[ct - c0];
                    row = ent + (ct - c0) * Ls;
                }
            } else {
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    if (t0 + u >= n) break;
                    int32_t s;
                    if (kMode == kModeLatent) s = __float2int_rn(__int_as_float(cur[u]) - __int_as_float(ch.x));
                    else s = cur[u];
                    int4 cs = ch;              // the symbol's row: the layout's ...
                    const uint4 *rs = row;
                    bool global = false;       // ... or one outside the group
                    if (kIdx && icur[u] != ct) {
                        flags |= kFlagNonChannel;
                        int c = icur[u];
                        if ((unsigned)c >= (unsigned)p.t.C) {
                            flags |= kFlagIndexRange;
                            c = 0;
                        }
                        if (c >= c0 && c < c0 + nc) {
                            cs = chan[c - c0];
                            rs = ent + (c - c0) * Ls;
                        } else {
                            global = true;
                            int32_t size = __ldg(p.t.sizes + c);
                            if (size < 2 || size > p.t.L) {
                                flags |= kFlagTable;
                                size = size < 2 ? 2 : p.t.L;
                            }
                            cs = make_int4(0, __ldg(p.t.offs + c), size - 2, c);
                        }
                    }
                    const int32_t value = (int32_t)((uint32_t)s - (uint32_t)cs.y);
                    const bool oor = (uint32_t)value >= (uint32_t)cs.z;
                    if (oor) {
                        const EscOut r = put_escape_call(x, escape_raw(value, cs.z), wrow, cap, j);
                        x = r.x;
                        j = r.j;
                    }
                    const int v = oor ? cs.z : value;
                    uint4 e;
                    if (kIdx && global) {
                        const int32_t *crow = p.t.cdfs + (int64_t)cs.w * p.t.L;
                        const uint32_t pe = pack_entry(__ldg(crow + v), __ldg(crow + v + 1), flags);
                        const uint32_t freq = (pe >> 16) + 1u;
                        const uint64_t m = g_magic[freq];
                        e = make_uint4((uint32_t)m, (uint32_t)(m >> 32), freq, pe & 0xFFFFu);
                    } else {
                        e = rs[v];
                    }
                    enc_step<true>(x, j, wrow, cap, e);
                    if (t0 + u + 1 < n) {  // step to the next symbol's channel only when one follows
                        rem -= kLanes;
                        if (rem < 0) {
                            do {
                                rem += p.HW;
                                --ct;
                            } while (rem < 0);
                            ch = chan[ct - c0];
                            row = ent + (ct - c0) * Ls;
                        }
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kB; ++u) {
                cur[u] = nxt[u];
                if (kIdx) icur[u] = inxt[u];
            }
        }
        // flush: the decoder reads the low word first
        if (n > 0) {
            if (j < cap) wrow[(int64_t)j * kLanes] = (uint32_t)(x >> 32);
            ++j;
            if (j < cap) wrow[(int64_t)j * kLanes] = (uint32_t)x;
            ++j;
        }
    }
    int rounds = j;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rounds = max(rounds, __shfl_xor_sync(0xffffffffu, rounds, o));
    p.used[chunk * kLanes + lane] = j;
    if (lane == 0) {
        p.rounds[chunk] = rounds;
        p.max_rounds_out[chunk] = (uint32_t)rounds;
    }
    if ((unsigned)rounds > my_max_used) my_max_used = (unsigned)rounds;
}

// Three CTAs of eight warps per SM (at most 85 registers a thread), so that
// a batch of 64 images at P_ch = 4 (384 groups) runs in one wave.
template <int kMode>
__global__ void __launch_bounds__(kThreads, 3) encode_lanes_kernel(EncParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t flags = 0;
    unsigned int my_max_used = 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int nbb = (p.B + W - 1) / W;
    const int64_t groups = (int64_t)p.K * nbb;
    const LanesSmem ls = lanes_smem(p.P, p.t.L, true);
    const uint4 *ent = reinterpret_cast<const uint4 *>(smem + ls.ent);
    const int4 *chan = reinterpret_cast<const int4 *>(smem + ls.chan);
    for (int64_t g = blockIdx.x; g < groups; g += gridDim.x) {
        const int k = (int)(g % p.K), bb = (int)(g / p.K);
        const int c0 = k * p.P, nc = min(p.P, p.t.C - c0);
        __syncthreads();  // the previous group's rows are no longer read
        stage_lanes<false>(p.t, c0, nc, true, smem, ls, kMode == kModeLatent ? p.medians : nullptr, flags);
        const int b = bb * W + warp;
        if (b < p.B)
            encode_lanes<kMode>(p, ent, chan, c0, nc, p.t.L - 1, (int64_t)b * p.K + k, lane, flags, my_max_used);
    }
    finish_encode(p, flags, my_max_used);
}

// One decode step (warp_ans_kernel.cu:219-329 semantics): the bucket of the
// slot names the symbol unless the slot lies past the bucket's first
// symbol, then a binary search over the rest of the bucket finds it.  The
// refill word is `cand` (word `word` of the lane's stream) and the one after
// it `cand2`: a refill moves `cand2` up and loads the next word, so each
// load has a whole renormalisation interval to arrive and steps without a
// refill load nothing.  Reads are clamped to the chunk's last round.
struct DecLane {
    uint64_t x;
    int word;
    uint32_t cand, cand2;
};

// cand / cand2 from the lane's stream at d.word (after an escape's reads)
__device__ __forceinline__ void dec_reload(DecLane &d, const uint32_t *__restrict__ base, int rm1) {
    d.cand = __ldg(base + (int64_t)min(d.word, rm1) * kLanes);
    d.cand2 = __ldg(base + (int64_t)min(d.word + 1, rm1) * kLanes);
}

__device__ __forceinline__ void dec_refill(DecLane &d, const uint32_t *__restrict__ base, int rm1) {
    const bool need = d.x < kRansL;
    d.x = need ? (d.x << 32) | (uint64_t)d.cand : d.x;
    if (need) {
        ++d.word;
        d.cand = d.cand2;
        d.cand2 = __ldg(base + (int64_t)min(d.word + 1, rm1) * kLanes);
    }
}

template <bool kPair>
__device__ __forceinline__ int32_t dec_step(DecLane &d, const uint2 *__restrict__ lrow, const uint32_t *__restrict__ row,
                                            int shift, int maxv, const uint32_t *__restrict__ base, int rm1) {
    const uint32_t slot = (uint32_t)d.x & 0xFFFFu;
    const uint2 le = lrow[slot >> shift];
    int32_t s;
    uint32_t st, endm1;
    if (kPair) {
        const uint32_t end0 = le.x >> 16;
        const bool more = slot > end0;
        s = (int32_t)(le.y >> 16) + (more ? 1 : 0);
        st = more ? end0 + 1u : (le.x & 0xFFFFu);
        endm1 = more ? (le.y & 0xFFFFu) : end0;
        if (more && slot > endm1) {  // three or more symbols in the bucket (or s0 is the last symbol)
            s = lanes_find(row, (int)(le.y >> 16), maxv, slot);
            const uint32_t e = row[s];
            st = e & 0xFFFFu;
            endm1 = e >> 16;
        }
    } else {
        uint32_t e = le.x;
        s = (int32_t)(le.y & 0xFFFFu);
        if (slot > (e >> 16)) {  // past the bucket's first symbol: search the rest of it
            s = lanes_find(row, s + 1, (int)(le.y >> 16), slot);
            e = row[s];
        }
        st = e & 0xFFFFu;
        endm1 = e >> 16;
    }
    const uint32_t freq = endm1 - st + 1u;
    d.x = (uint64_t)freq * (d.x >> 16) + (uint64_t)(int64_t)(int32_t)(slot - st);
    dec_refill(d, base, rm1);
    return s;
}

// dec_step for a row outside the staged group (explicit indexes): a binary
// search of the row's CDF in global memory, the full-table decode's lookup.
__device__ __forceinline__ int32_t dec_step_global(DecLane &d, const TableArgs &t, int c, int maxv,
                                                   const uint32_t *__restrict__ base, int rm1, uint32_t &flags) {
    const uint32_t slot = (uint32_t)d.x & 0xFFFFu;
    const int32_t *row = t.cdfs + (int64_t)c * t.L;
    int lo = 0, hi = maxv;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((uint32_t)__ldg(row + mid + 1) > slot) hi = mid;
        else lo = mid + 1;
    }
    const uint32_t e = pack_entry(__ldg(row + lo), __ldg(row + lo + 1), flags);
    const uint32_t st = e & 0xFFFFu, freq = (e >> 16) + 1u;
    d.x = (uint64_t)freq * (d.x >> 16) + (uint64_t)(int64_t)(int32_t)(slot - st);
    dec_refill(d, base, rm1);
    return lo;
}

// Escape decode inlined into the decode loop (warp_ans_kernel.cu:308-325):
// the count nibbles, then the value nibbles low to high.  Words are read
// straight from the lane's stream, bounded by its rounds; returns false on
// a corrupt stream (more than 8 value nibbles, or words past the rounds).
__device__ __forceinline__ bool dec_escape(DecLane &d, const uint32_t *__restrict__ base, int rounds, int32_t maxv,
                                           int32_t &value) {
    bool bad = false;
    auto nibble = [&]() -> uint32_t {
        const uint32_t v = (uint32_t)d.x & kBypassMax;
        d.x >>= kBypassBits;
        if (d.x < kRansL) {
            uint32_t w = 0u;
            if (d.word < rounds) w = __ldg(base + (int64_t)d.word * kLanes);
            else bad = true;
            ++d.word;
            d.x = (d.x << 32) | (uint64_t)w;
        }
        return v;
    };
    uint32_t v = nibble();
    uint32_t n_bypass = v;
    while (v == kBypassMax && !bad && n_bypass <= 8u) {
        v = nibble();
        n_bypass += v;
    }
    if (n_bypass > 8u || bad) return false;
    uint32_t raw = 0;
    for (uint32_t i = 0; i < n_bypass; ++i) raw |= nibble() << (i * kBypassBits);
    int32_t val = (int32_t)raw >> 1;  // int32 arithmetic shift, as in the reference
    if (raw & 1u) val = -val - 1;
    else val = (int32_t)((uint32_t)val + (uint32_t)maxv);
    value = val;
    return !bad;
}

// Decodes one chunk: each lane reads its state, then its symbols first to
// last, eight at a time (one vote and one bookkeeping step per eight
// symbols: about 2% faster than four).  A group of eight symbols in one
// channel (every group when HW is a multiple of 256) has no channel
// bookkeeping; the ragged end and groups that cross a channel step per
// symbol.  A lane that
// consumes more words than its chunk holds marks the payload corrupt.
//
// With explicit indexes (kModeIdx) a group also needs its indexes to be the
// channel layout (warp vote); otherwise it steps per symbol, and a symbol
// whose row lies outside the staged group searches that row in global
// memory.
template <int kMode, bool kPair>
__device__ __forceinline__ void decode_lanes(const DecParams &p, const uint32_t *__restrict__ ent,
                                             const int4 *__restrict__ chan, const uint2 *__restrict__ lut, int shift,
                                             int c0, int nc, int Ls, int64_t chunk, int lane, uint32_t &flags) {
    constexpr int kG = 8;
    constexpr bool kIdx = kMode == kModeIdx;
    const uint32_t *body = reinterpret_cast<const uint32_t *>(p.packed + p.header_bytes);
    const int b = (int)(chunk / p.K);
    const int k = (int)(chunk - (int64_t)b * p.K);
    const int64_t start64 = (int64_t)k * p.chunk_len;
    if (start64 >= p.N) return;
    const int start = (int)start64;
    const int end = (int)min(start64 + p.chunk_len, (int64_t)p.N);
    uint64_t off;
    if (p.offsets) {
        off = p.offsets[chunk];
    } else {
        uint64_t sum = 0;
        for (int64_t c = lane; c < chunk; c += kLanes) sum += (uint64_t)__ldg(p.max_rounds + c);
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        off = sum * kLanes;
    }
    const int rounds = (int)__ldg(p.max_rounds + chunk);
    if (rounds < 2 || rounds > 0x7fffffff - 8) {
        flags |= kFlagCorrupt;
        return;
    }
    const int first = start + lane;
    const int n = first < end ? (end - 1 - first) / kLanes + 1 : 0;
    const uint32_t *base = body + off + lane;
    const int rm1 = rounds - 1;
    // the chunk's stream into L2, one row per lane and step
    for (int r = lane; r < rounds; r += kLanes) asm volatile("prefetch.global.L2 [%0];" ::"l"(body + off + (int64_t)r * kLanes));
    // every lane runs the same number of groups (the warp's longest), so
    // that the warp votes below always see all 32 lanes; a lane past its
    // own symbols takes the guarded path and does nothing
    int nmax = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, o));
    if (nmax == 0) return;
    DecLane d;
    d.x = (uint64_t)__ldg(base) | ((uint64_t)__ldg(base + kLanes) << 32);
    d.word = 2;
    dec_reload(d, base, rm1);
    int ct = n > 0 ? first / p.HW : c0, rem = n > 0 ? first - ct * p.HW : 0;
    int4 ch = chan[ct - c0];
    const uint32_t *row = ent + (ct - c0) * Ls;
    const uint2 *lrow = lut + (int64_t)(ct - c0) * (65536 >> shift);
    const int64_t pos0 = (int64_t)b * p.N + first;
    int32_t *orow = kMode == kModeLatent ? nullptr : p.out + pos0;
    float *yrow = kMode == kModeLatent ? p.y_out + pos0 : nullptr;
    const int32_t *irow = kIdx ? p.idx + pos0 : nullptr;
    int32_t icur[kIdx ? kG : 1], inxt[kIdx ? kG : 1];
    if (kIdx) {
#pragma unroll
        for (int u = 0; u < kG; ++u) icur[u] = u < n ? __ldg(irow + (int64_t)u * kLanes) : 0;
    }
    bool bad = false;
    auto finish_symbol = [&](int32_t s, int t) {
        const bool esc = s == ch.z;
        if (__any_sync(0xffffffffu, esc)) {  // some lane escapes: its value follows as bypass nibbles
            if (esc) {
                bad |= !dec_escape(d, base, rounds, ch.z, s);
                dec_reload(d, base, rm1);
            }
        }
        const int32_t sym = (int32_t)((uint32_t)s + (uint32_t)ch.y);
        if (kMode == kModeLatent) yrow[(int64_t)t * kLanes] = __int2float_rn(sym) + __int_as_float(ch.x);
        else orow[(int64_t)t * kLanes] = sym;
    };
    // cs: the symbol's row ({median, offset, maxv}); ch unless an explicit
    // index names another row
    auto finish_symbol_guarded = [&](int32_t s, int t, bool live, const int4 &cs) {
        const bool esc = live && s == cs.z;
        if (__any_sync(0xffffffffu, esc)) {
            if (esc) {
                bad |= !dec_escape(d, base, rounds, cs.z, s);
                dec_reload(d, base, rm1);
            }
        }
        if (live) {
            const int32_t sym = (int32_t)((uint32_t)s + (uint32_t)cs.y);
            if (kMode == kModeLatent) yrow[(int64_t)t * kLanes] = __int2float_rn(sym) + __int_as_float(cs.x);
            else orow[(int64_t)t * kLanes] = sym;
        }
    };
    auto next_channel = [&]() {
        do {
            rem -= p.HW;
            ++ct;
        } while (rem >= p.HW);
        ch = chan[ct - c0];
        row = ent + (ct - c0) * Ls;
        lrow = lut + (int64_t)(ct - c0) * (65536 >> shift);
    };
    for (int t = 0; t < nmax; t += kG) {
        asm volatile("prefetch.global.L1 [%0];" ::"l"(base + (int64_t)min(d.word + 6, rm1) * kLanes));
        bool one_channel = t + kG <= n && rem + (kG - 1) * kLanes < p.HW;
        if (kIdx) {
#pragma unroll
            for (int u = 0; u < kG; ++u) {
                one_channel = one_channel && icur[u] == ct;
                inxt[u] = t + kG + u < n ? __ldg(irow + (int64_t)(t + kG + u) * kLanes) : 0;
            }
        }
        if (__all_sync(0xffffffffu, one_channel)) {
#pragma unroll
            for (int u = 0; u < kG; ++u) finish_symbol(dec_step<kPair>(d, lrow, row, shift, ch.z, base, rm1), t + u);
            rem += kG * kLanes;
            if (rem >= p.HW && t + kG < n) next_channel();
        } else {
            // lanes past their last symbol keep voting but do nothing
#pragma unroll
            for (int u = 0; u < kG; ++u) {
                const bool live = t + u < n;
                int32_t s = 0;
                int4 cs = ch;
                if (kIdx && live && icur[u] != ct) {
                    flags |= kFlagNonChannel;
                    int c = icur[u];
                    if ((unsigned)c >= (unsigned)p.t.C) {
                        flags |= kFlagIndexRange;
                        c = 0;
                    }
                    if (c >= c0 && c < c0 + nc) {
                        cs = chan[c - c0];
                        s = dec_step<kPair>(d, lut + (int64_t)(c - c0) * (65536 >> shift), ent + (c - c0) * Ls, shift,
                                            cs.z, base, rm1);
                    } else {
                        int32_t size = __ldg(p.t.sizes + c);
                        if (size < 2 || size > p.t.L) {
                            flags |= kFlagTable;
                            size = size < 2 ? 2 : p.t.L;
                        }
                        cs = make_int4(0, __ldg(p.t.offs + c), size - 2, 0);
                        s = dec_step_global(d, p.t, c, cs.z, base, rm1, flags);
                    }
                } else if (live) {
                    s = dec_step<kPair>(d, lrow, row, shift, ch.z, base, rm1);
                }
                finish_symbol_guarded(s, t + u, live, cs);
                if (live) {
                    rem += kLanes;
                    if (rem >= p.HW && t + u + 1 < n) next_channel();
                }
            }
        }
        if (kIdx) {
#pragma unroll
            for (int u = 0; u < kG; ++u) icur[u] = inxt[u];
        }
    }
    if (n > 0 && (bad || d.word > rounds)) flags |= kFlagCorrupt;
}

template <int kMode, bool kPair>
__global__ void __launch_bounds__(kThreads) decode_lanes_kernel(DecParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_skip;
    uint32_t flags = 0;
    if (threadIdx.x == 0) s_skip = decode_skip(p) ? 1 : 0;
    __syncthreads();
    const bool skip = s_skip != 0;
    // W warps decode a group's W images; a CTA of fewer images than kWarps
    // launches kWarps warps anyway, and the rest help stage the group's rows
    // and bucket tables
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = p.group_warps;
    const int P = p.chunk_len / p.HW;
    const int nbb = (p.B + W - 1) / W;
    const int64_t groups = (int64_t)p.K * nbb;
    const LanesSmem ls = lanes_smem(P, p.t.L, false);
    const uint32_t *ent = reinterpret_cast<const uint32_t *>(smem + ls.ent);
    const int4 *chan = reinterpret_cast<const int4 *>(smem + ls.chan);
    const uint2 *lut = reinterpret_cast<const uint2 *>(smem + ls.lut);
    for (int64_t g = blockIdx.x; g < groups && !skip; g += gridDim.x) {
        const int k = (int)(g % p.K), bb = (int)(g / p.K);
        const int c0 = min(k * P, p.t.C), nc = max(0, min(P, p.t.C - c0));
        __syncthreads();
        stage_lanes<kPair>(p.t, c0, nc, false, smem, ls, kMode == kModeLatent ? p.medians : nullptr, flags);
        // an invalid row leaves buckets unfilled: decode nothing (the table
        // error is reported)
        if (__syncthreads_or((int)(flags & kFlagTable))) continue;
        const int b = bb * W + warp;
        if (warp < W && b < p.B)
            decode_lanes<kMode, kPair>(p, ent, chan, lut, ls.lut_shift, c0, nc, p.t.L - 1, (int64_t)b * p.K + k,
                                       lane, flags);
    }
    finish_decode(p, flags);
}

// Pack with coalesced reads: a warp reads its chunk's staging rows in
// emission order, 128 bytes a row, and each lane stores word j of its
// stream at row used - 1 - j of the payload (its decode order); rows from
// used to max_rounds hold zeros.  Stores scatter over the chunk's rows and
// merge in L2.  Several warps share a chunk when chunks are few.
__global__ void __launch_bounds__(kThreads) pack_rows_kernel(PackParams p, int split) {
    const long long total_words = p.ctrl->status[kStTotalWords];
    const int rows_cap = (int)p.ctrl->status[kStRowsCap];
    if (p.header_bytes + 4 * (int64_t)total_words != p.packed_bytes) return;  // not the last encode's size
    uint32_t *hdr = reinterpret_cast<uint32_t *>(p.packed);
    if (blockIdx.x == 0 && threadIdx.x < 8) {
        uint32_t h = 0;
        switch (threadIdx.x) {
            case 0: h = (uint32_t)p.N; break;
            case 1: h = (uint32_t)p.chunk_len; break;
            case 2: h = ((uint32_t)p.K & 0xFFFFu) | (((uint32_t)p.B & 0xFFFFu) << 16); break;
            case 3: h = 2u | (32u << 16); break;
            default: h = 0u;
        }
        hdr[threadIdx.x] = h;
    }
    const int64_t table_end = 32 + 4 * p.chunks;
    if (blockIdx.x == 0 && threadIdx.x >= 8 && threadIdx.x < 8 + (p.header_bytes - table_end) / 4)
        hdr[table_end / 4 + (threadIdx.x - 8)] = 0u;
    const int lane = threadIdx.x & 31;
    uint32_t *body = reinterpret_cast<uint32_t *>(p.packed + p.header_bytes);
    const int64_t tasks = p.chunks * split;
    const int64_t warp_stride = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks;
         task += warp_stride) {
        const int64_t chunk = task / split;
        const int part = (int)(task - chunk * split);
        const int rounds = __ldg(p.rounds + chunk);
        int used = __ldg(p.used + chunk * kLanes + lane);
        if (used > rows_cap) used = 0;  // overflowed staging: never packed by the host
        if (lane == 0 && part == 0) hdr[8 + chunk] = (uint32_t)rounds;
        const uint32_t *st = p.stage + chunk * (int64_t)rows_cap * kLanes + lane;
        uint32_t *out = body + p.offsets[chunk] + lane;
        const int per = (rounds + split - 1) / split;
        const int j0 = part * per, j1 = min(rounds, j0 + per);
        int j = j0;
        for (; j + 8 <= j1; j += 8) {
            uint32_t v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = j + i < rows_cap ? __ldcs(st + (int64_t)(j + i) * kLanes) : 0u;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int jj = j + i;
                const bool word = jj < used;
                out[(int64_t)(word ? used - 1 - jj : jj) * kLanes] = word ? v[i] : 0u;
            }
        }
        for (; j < j1; ++j) {
            const bool word = j < used;
            out[(int64_t)(word ? used - 1 - j : j) * kLanes] = word ? st[(int64_t)j * kLanes] : 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static std::mutex g_init_mutex;
static bool g_magic_ready[64];

// ---- status read-back without the copy engines -----------------------------
// The encode's size / status words and the decode's check flags come back
// through a 64-byte pinned host buffer mapped into the device's address space
// (one per device and stream): a one-warp kernel stores them there, and the
// host waits for the stream only.  A cudaMemcpy of those few bytes would be
// queued on a copy engine behind whatever bulk transfers other streams have
// issued (a batch's upload or download), and the host would wait for those.
// Two slots: [0, 8) for the synchronous read-backs, [8, 16) for the status
// of a submitted encode (fcai_warp_div_encode_latent_submit), which the host
// collects later in fcai_warp_div_encode_finish by waiting on `done` alone.
struct MappedStatus {
    volatile long long *host;
    long long *dev;
    cudaEvent_t done;
    int *pending;  // a submitted encode awaits its finish (shared flag)
};
static std::mutex g_status_mutex;
static std::unordered_map<uint64_t, MappedStatus> g_status;

__global__ void status_to_host_kernel(const long long *__restrict__ src, long long *dst, int n) {
    if ((int)threadIdx.x < n) dst[threadIdx.x] = src[threadIdx.x];
}

static int mapped_status(cudaStream_t stream, MappedStatus *out) {
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t key = ((uint64_t)(uint32_t)dev << 48) ^ reinterpret_cast<uint64_t>(stream);
    std::lock_guard<std::mutex> lock(g_status_mutex);
    auto it = g_status.find(key);
    if (it != g_status.end()) {
        *out = it->second;
        return FCAI_OK;
    }
    void *h = nullptr;
    void *d = nullptr;
    FCAI_CUDA_TRY(cudaHostAlloc(&h, 128, cudaHostAllocMapped | cudaHostAllocPortable));
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess || !d) {
        cudaFreeHost(h);
        return fcai::fail(FCAI_ERR_CUDA, "mapped status buffer has no device address");
    }
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        cudaFreeHost(h);
        return fcai::fail(FCAI_ERR_CUDA, "status event creation failed");
    }
    MappedStatus m{static_cast<volatile long long *>(h), static_cast<long long *>(d), ev, new int(0)};
    g_status.emplace(key, m);
    *out = m;
    return FCAI_OK;
}

// Reads n (<= 8) status words of the control block after the stream's
// queued work.
static int read_status(const long long *src, int n, cudaStream_t stream, long long *out) {
    MappedStatus m{};
    if (int rc = mapped_status(stream, &m)) return rc;
    status_to_host_kernel<<<1, 32, 0, stream>>>(src, m.dev, n);
    FCAI_CUDA_TRY(cudaGetLastError());
    FCAI_CUDA_TRY(cudaStreamSynchronize(stream));
    for (int i = 0; i < n; ++i) out[i] = m.host[i];
    return FCAI_OK;
}

// ---- payload transfers without the copy engines -----------------------------
// Copies between device memory and pinned host memory that is mapped into the
// device's address space, done by SM loads and stores over PCIe, for the same
// reason: a small payload must not wait behind a batch's bulk copies.
__global__ void copy16_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int64_t n16) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}
__global__ void copy1_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// The device address of p: device memory as is, host memory only if it is
// pinned and mapped (nullptr otherwise, and for memory of another device).
static void *device_address(const void *p, int dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return a.device == dev ? a.devicePointer : nullptr;
    if (a.type == cudaMemoryTypeHost) return a.devicePointer;
    return nullptr;
}

static int ensure_magic(cudaStream_t stream) {
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fcai::fail(FCAI_ERR_CUDA, "device ordinal %d unsupported", dev);
    std::lock_guard<std::mutex> lock(g_init_mutex);
    if (g_magic_ready[dev]) return FCAI_OK;
    init_magic_kernel<<<(65537 + 255) / 256, 256, 0, stream>>>();
    FCAI_CUDA_TRY(cudaGetLastError());
    FCAI_CUDA_TRY(cudaStreamSynchronize(stream));
    g_magic_ready[dev] = true;
    return FCAI_OK;
}

struct Dims {
    int B, N, C, P, K, chunk_len, HW;
    int64_t chunks, header_bytes;
};

static int make_dims(int32_t B, int32_t N, int32_t C, int32_t P, Dims &d) {
    // warp_ans_kernel_v2.cu:198-203
    if (B <= 0 || N <= 0 || C <= 0) return fcai::fail(FCAI_ERR_INVALID, "empty/invalid coder input dimensions");
    if (N % C != 0)
        return fcai::fail(FCAI_ERR_INVALID, "WarpANS currently requires symbols per batch divisible by CDF count");
    if (P <= 0 || P > C) return fcai::fail(FCAI_ERR_INVALID, "P_ch must be in [1, C]");
    if (B > 65535 || C > 65535) return fcai::fail(FCAI_ERR_INVALID, "B/C exceed WarpANS header field capacity");
    if ((int64_t)N * C >= INT32_MAX) return fcai::fail(FCAI_ERR_INVALID, "coder dimensions exceed kernel index range");
    d.B = B;
    d.N = N;
    d.C = C;
    d.P = P;
    d.HW = N / C;
    d.K = (C + P - 1) / P;
    d.chunk_len = P * d.HW;
    d.chunks = (int64_t)B * d.K;
    if (d.chunks > INT32_MAX) return fcai::fail(FCAI_ERR_INVALID, "B * K exceeds the header's int32 range");
    d.header_bytes = (32 + 4 * d.chunks + 15) & ~int64_t(15);
    return FCAI_OK;
}

static inline int64_t rows_worst(const Dims &d) {
    return (int64_t)kMaxSymbolWords * ((d.chunk_len + kLanes - 1) / kLanes) + 2;
}

static int64_t encode_smem_bytes(int C, int L) { return (((int64_t)C * (L - 1) * 4 + 15) & ~15ll) + (int64_t)C * 8; }
static int64_t decode_smem_bytes(int C, int L) {
    return encode_smem_bytes(C, L) + (int64_t)C * kLutBuckets * 2;
}

// Per (kernel, device) launch shape: the dynamic shared memory opt-in is
// raised to the largest size seen and the occupancy is queried once per
// distinct size, so repeated calls do no driver queries.
struct LaunchCache {
    const void *fn;
    int dev;
    int64_t smem_optin;
    int64_t smem_last;
    int warps_last;
    int occ_last;
};
static std::mutex g_launch_mutex;
static LaunchCache g_launch[64];
static int g_launch_n = 0;

// Warps per CTA: 8, unless there are too few chunks to give every SM two
// CTAs' worth, in which case smaller CTAs spread the chunks over more SMs.
static int warps_for(int64_t chunks) {
    const int64_t sms = fcai::sm_count();
    int w = kWarps;
    while (w > 1 && chunks < (int64_t)w * sms * 2) w >>= 1;
    return w;
}

template <typename K>
static int grid_for(K kernel, int64_t smem, int64_t chunks, int warps, int &grid) {
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(g_launch_mutex);
        LaunchCache *e = nullptr;
        for (int i = 0; i < g_launch_n; ++i)
            if (g_launch[i].fn == (const void *)kernel && g_launch[i].dev == dev) e = &g_launch[i];
        if (!e && g_launch_n < 64) {
            e = &g_launch[g_launch_n++];
            *e = LaunchCache{(const void *)kernel, dev, 48 * 1024, -1, 0, 0};
        }
        if (e && e->smem_last == smem && e->warps_last == warps) {
            occ = e->occ_last;
        } else {
            if (smem > (e ? e->smem_optin : 48 * 1024)) {
                FCAI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                if (e) e->smem_optin = smem;
            }
            FCAI_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, warps * kLanes, (size_t)smem));
            if (e) {
                e->smem_last = smem;
                e->warps_last = warps;
                e->occ_last = occ;
            }
        }
    }
    if (occ < 1) occ = 1;
    int64_t want = (chunks + warps - 1) / warps;
    int64_t cap = (int64_t)fcai::sm_count() * occ;
    grid = (int)(want < cap ? want : cap);
    if (grid < 1) grid = 1;
    return FCAI_OK;
}

// Warps per CTA for chunk groups: up to 8 images per group, fewer when that
// leaves SMs idle (few chunks per image, e.g. large P).
static int group_warps(int B, int K) {
    const int64_t sms = fcai::sm_count();
    int w = B < kWarps ? B : kWarps;
    while (w > 1 && (int64_t)K * ((B + w - 1) / w) < sms) w >>= 1;
    return w < 1 ? 1 : w;
}

template <bool kSmem>
static int launch_encode_full(const EncParams &p, int64_t smem, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = warps_for(p.chunks);
    if ((rc = grid_for(encode_kernel<kSmem>, kSmem ? smem : 0, p.chunks, warps, grid))) return rc;
    encode_kernel<kSmem><<<grid, warps * kLanes, kSmem ? smem : 0, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

template <int kMode>
static int launch_encode_group(const EncParams &p, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = group_warps(p.B, p.K);
    const int64_t groups = (int64_t)p.K * ((p.B + warps - 1) / warps);
    if ((rc = grid_for(encode_group_kernel<kMode>, 0, groups * warps, warps, grid))) return rc;
    encode_group_kernel<kMode><<<grid, warps * kLanes, 0, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

template <int kMode, bool kSmem>
static int launch_decode_full(const DecParams &p, int64_t smem, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = warps_for(p.chunks);
    if ((rc = grid_for(decode_kernel<kMode, kSmem>, kSmem ? smem : 0, p.chunks, warps, grid))) return rc;
    decode_kernel<kMode, kSmem><<<grid, warps * kLanes, kSmem ? smem : 0, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

template <int kMode>
static int launch_encode_lanes(const EncParams &p, int64_t smem, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = group_warps(p.B, p.K);
    const int64_t groups = (int64_t)p.K * ((p.B + warps - 1) / warps);
    if ((rc = grid_for(encode_lanes_kernel<kMode>, smem, groups * warps, warps, grid))) return rc;
    encode_lanes_kernel<kMode><<<grid, warps * kLanes, smem, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

template <int kMode, bool kPair>
static int launch_decode_lanes(DecParams p, int64_t smem, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = group_warps(p.B, p.K);
    p.group_warps = warps;
    const int64_t groups = (int64_t)p.K * ((p.B + warps - 1) / warps);
    // grid sized as for one warp per image; every CTA has kWarps warps
    if ((rc = grid_for(decode_lanes_kernel<kMode, kPair>, smem, groups * kWarps, kWarps, grid))) return rc;
    decode_lanes_kernel<kMode, kPair><<<grid, kThreads, smem, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

template <int kMode>
static int launch_decode_group(const DecParams &p, cudaStream_t stream) {
    int grid = 1, rc;
    const int warps = group_warps(p.B, p.K);
    const int64_t groups = (int64_t)p.K * ((p.B + warps - 1) / warps);
    if ((rc = grid_for(decode_group_kernel<kMode>, 0, groups * warps, warps, grid))) return rc;
    decode_group_kernel<kMode><<<grid, warps * kLanes, 0, stream>>>(p);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

static int check_tables_args(const int32_t *cdfs, int32_t C, int32_t L, const int32_t *sizes, const int32_t *offs) {
    if (!cdfs || !sizes || !offs) return fcai::fail(FCAI_ERR_INVALID, "null CDF table pointer");
    if (L < 2) return fcai::fail(FCAI_ERR_INVALID, "CDF table cannot be empty");
    if ((int64_t)C * L >= INT32_MAX) return fcai::fail(FCAI_ERR_INVALID, "CDF table too large");
    return FCAI_OK;
}

static int flags_to_status(long long flags, bool encode) {
    if (flags & kFlagIndexRange) return fcai::fail(FCAI_ERR_INDEX_RANGE, "indexes contain a value outside the CDF table range");
    if (flags & kFlagTable)
        return fcai::fail(FCAI_ERR_TABLE,
                          "CDF table invalid: cdf_sizes must lie in [2, L] and each row must be strictly "
                          "increasing within [0, 65536]");
    if (!encode) {
        if (flags & kFlagHeader)
            return fcai::fail(FCAI_ERR_HEADER, "warp_div packed header is inconsistent with payload metadata");
        if (flags & kFlagRounds)
            return fcai::fail(FCAI_ERR_ROUNDS, "warp_div packed header round counts do not match payload metadata");
        if (flags & kFlagCorrupt)
            return fcai::fail(FCAI_ERR_CORRUPT, "warp_div payload body is inconsistent with its chunk rounds");
    }
    return FCAI_OK;
}

// Encode scratch of fcai_warp_div_encode_noalloc.  Module-scope __device__
// storage exists once in each device's context from the moment this library's
// module is loaded there, so that entry point needs no device allocation.
// Every call on a device shares it (see the header on overlapping calls).
constexpr int64_t kScratchBytes = FCAI_WARP_DIV_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_encode_scratch[kScratchBytes];

static std::mutex g_scratch_mutex;
static void *g_scratch_ptr[64];

// Device address of g_encode_scratch on the current device: looked up once
// per device, with that device current, and cached.
static int encode_scratch(void **out) {
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fcai::fail(FCAI_ERR_CUDA, "device ordinal %d unsupported", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void *ptr = nullptr;
        FCAI_CUDA_TRY(cudaGetSymbolAddress((void **)&ptr, g_encode_scratch));
        if (!ptr) return fcai::fail(FCAI_ERR_CUDA, "cudaGetSymbolAddress returned a null scratch address");
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return FCAI_OK;
}

// Shared body of the encode entry points.
// The encode's size and status from its status words (kSt* slots).
static int encode_info_from_status(const Dims &d, const EncLayout &el, const long long *status,
                                   int64_t workspace_bytes, fcai_warp_div_encode_info *info) {
    const long long flags = status[kStFlags];
    info->header_bytes = d.header_bytes;
    info->chunk_len = d.chunk_len;
    info->p_ch = d.P;
    info->index_layout_is_channel = (flags & kFlagNonChannel) ? 0 : 1;
    info->packed_bytes = d.header_bytes + 4 * (int64_t)status[kStTotalWords];
    info->required_workspace_bytes = el.fixed_bytes + d.chunks * (int64_t)status[kStMaxUsed] * kLanes * 4;
    if (int rc = flags_to_status(flags, true)) return rc;
    if (flags & kFlagOverflow)
        return fcai::fail(FCAI_ERR_WORKSPACE, "encode staging needs %lld workspace bytes, %lld given",
                          (long long)info->required_workspace_bytes, (long long)workspace_bytes);
    return FCAI_OK;
}

// How an encode returns its status words to the host.
enum class StatusPath {
    kMapped,  // the encode's last CTA writes the stream's mapped pinned slot, then a stream wait
    kSubmit,  // as kMapped into the second slot, collected by fcai_warp_div_encode_finish
    kCopy,    // cudaMemcpyAsync into the caller's stack, then a stream wait: creates
              // nothing (no pinned slot, no event) on any call
};

// kSubmit: enqueue the encode and the copy of its status words to the mapped
// buffer's second slot, record the stream's status event and return at once
// (info untouched); fcai_warp_div_encode_finish collects the status.
static int encode_impl(int mode, const int32_t *symbols, const int32_t *indexes, const float *y,
                       const float *medians, int32_t B, int32_t N, const int32_t *cdfs, int32_t C, int32_t L,
                       const int32_t *cdf_sizes, const int32_t *offsets, int32_t P, void *workspace,
                       int64_t workspace_bytes, uint32_t *max_rounds, fcai_warp_div_encode_info *info,
                       cudaStream_t stream, StatusPath path = StatusPath::kMapped) {
    const bool submit = path == StatusPath::kSubmit;
    Dims d;
    int rc = make_dims(B, N, C, P, d);
    if (rc) return rc;
    if ((rc = check_tables_args(cdfs, C, L, cdf_sizes, offsets))) return rc;
    if (!workspace || !max_rounds || (!info && !submit)) return fcai::fail(FCAI_ERR_INVALID, "null argument");
    MappedStatus ms{};
    if (path != StatusPath::kCopy) {
        if ((rc = mapped_status(stream, &ms))) return rc;
        if (*ms.pending)
            return fcai::fail(FCAI_ERR_INVALID,
                              "an encode submitted on this stream awaits fcai_warp_div_encode_finish");
    }
    if (mode == kModeLatent ? (!y || !medians) : !symbols) return fcai::fail(FCAI_ERR_INVALID, "null input");
    EncLayout el = enc_layout(d.chunks);
    int64_t avail = workspace_bytes - el.fixed_bytes;
    int64_t rows_cap = avail > 0 ? avail / (d.chunks * kLanes * 4) : 0;
    if (rows_cap > rows_worst(d)) rows_cap = rows_worst(d);
    if (rows_cap < 2) {
        if (info) info->required_workspace_bytes = el.fixed_bytes + d.chunks * rows_worst(d) * kLanes * 4;
        return fcai::fail(FCAI_ERR_WORKSPACE, "encode workspace of %lld bytes is too small",
                          (long long)workspace_bytes);
    }
    if ((rc = ensure_magic(stream))) return rc;

    uint8_t *ws = static_cast<uint8_t *>(workspace);
    EncParams p;
    p.sym = symbols;
    p.idx = indexes;
    p.y = y;
    p.medians = medians;
    p.t = TableArgs{cdfs, cdf_sizes, offsets, C, L};
    p.B = d.B;
    p.N = d.N;
    p.P = d.P;
    p.K = d.K;
    p.chunk_len = d.chunk_len;
    p.HW = d.HW;
    p.rows_cap = (int)rows_cap;
    p.chunks = d.chunks;
    p.ctrl = reinterpret_cast<Control *>(ws);
    p.rounds = reinterpret_cast<int32_t *>(ws + el.rounds);
    p.used = reinterpret_cast<int32_t *>(ws + el.used);
    p.offsets = reinterpret_cast<unsigned long long *>(ws + el.offsets);
    p.stage = reinterpret_cast<uint32_t *>(ws + el.stage);
    p.max_rounds_out = max_rounds;
    // the last CTA writes the status words to the stream's mapped slot itself
    // (no copy kernel); the no-allocation path copies them with the stream
    p.status_out = path == StatusPath::kCopy ? nullptr : (submit ? ms.dev + 8 : ms.dev);

    // the group's rows in shared memory (every P of the reference's sweep
    // with 16-bit CDFs of <= 66 entries), else global tables; explicit
    // indexes outside the group's rows read theirs from global memory
    const int64_t smem = lanes_smem(d.P, L, true).bytes;
    if (smem <= kMaxSmemBytes) {
        rc = mode == kModeIdx       ? launch_encode_lanes<kModeIdx>(p, smem, stream)
             : mode == kModeChannel ? launch_encode_lanes<kModeChannel>(p, smem, stream)
                                    : launch_encode_lanes<kModeLatent>(p, smem, stream);
    } else if (mode == kModeIdx) {
        const int64_t full = encode_smem_bytes(C, L);
        rc = full <= kMaxSmemBytes ? launch_encode_full<true>(p, full, stream) : launch_encode_full<false>(p, full, stream);
    } else {
        rc = mode == kModeChannel ? launch_encode_group<kModeChannel>(p, stream)
                                  : launch_encode_group<kModeLatent>(p, stream);
    }
    if (rc) return rc;
    if (submit) {
        FCAI_CUDA_TRY(cudaEventRecord(ms.done, stream));
        *ms.pending = 1;
        return FCAI_OK;
    }
    long long status[8];
    if (path == StatusPath::kCopy) {
        FCAI_CUDA_TRY(cudaMemcpyAsync(status, p.ctrl->status, sizeof(status), cudaMemcpyDeviceToHost, stream));
        FCAI_CUDA_TRY(cudaStreamSynchronize(stream));
    } else {
        FCAI_CUDA_TRY(cudaStreamSynchronize(stream));
        for (int i = 0; i < 8; ++i) status[i] = ms.host[i];
    }
    return encode_info_from_status(d, el, status, workspace_bytes, info);
}

// Unchecked decodes up to this many chunks sum their offsets in the decode
// kernel (at most 64 loads per lane) instead of launching the prep kernel.
constexpr int64_t kInlineOffsetChunks = 2048;

// Shared body of the decode entry points.
static int decode_impl(int mode, const uint8_t *packed, int64_t packed_bytes, const uint32_t *max_rounds, int32_t K,
                       int64_t header_bytes, int32_t chunk_len, const int32_t *indexes, int32_t B, int32_t N,
                       const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets,
                       const float *medians, int32_t *symbols_out, float *y_out, void *workspace,
                       int64_t workspace_bytes, int32_t check, int32_t *index_layout_is_channel,
                       cudaStream_t stream) {
    // warp_ans_kernel.cu:489-503
    if (B <= 0 || N <= 0 || C <= 0 || N % C != 0)
        return fcai::fail(FCAI_ERR_INVALID, "invalid decode dimensions/channel layout");
    if (K <= 0 || header_bytes < 32 || chunk_len <= 0) return fcai::fail(FCAI_ERR_INVALID, "invalid payload metadata");
    if (header_bytes >= packed_bytes) return fcai::fail(FCAI_ERR_INVALID, "header exceeds packed payload size");
    int rc = check_tables_args(cdfs, C, L, cdf_sizes, offsets);
    if (rc) return rc;
    if (!packed || !max_rounds || !workspace) return fcai::fail(FCAI_ERR_INVALID, "null argument");
    if (mode == kModeLatent ? (!medians || !y_out) : !symbols_out) return fcai::fail(FCAI_ERR_INVALID, "null output");
    const int64_t chunks = (int64_t)B * K;
    if (chunks > INT32_MAX) return fcai::fail(FCAI_ERR_INVALID, "B * K exceeds the header's int32 range");
    // coders/warp_div.py:56-61 (structure of the payload sizes)
    if (header_bytes % 16 || header_bytes < 32 + 4 * chunks)
        return fcai::fail(FCAI_ERR_INVALID, "warp_div header size does not match chunk metadata");
    if (packed_bytes % 4) return fcai::fail(FCAI_ERR_INVALID, "warp_div packed payload must be uint32 aligned");
    DecLayout dl = dec_layout(chunks);
    if (workspace_bytes < dl.fixed_bytes)
        return fcai::fail(FCAI_ERR_WORKSPACE, "decode workspace needs %lld bytes", (long long)dl.fixed_bytes);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    Control *ctrl = reinterpret_cast<Control *>(ws);
    unsigned long long *offs = reinterpret_cast<unsigned long long *>(ws + dl.offsets);

    // Unchecked decodes of few chunks (payloads whose header the caller has
    // validated on the host) need no prep launch: each warp sums its chunk's
    // offset itself.  Otherwise the prep kernel checks the header and scans.
    const bool prep = check || chunks > kInlineOffsetChunks;
    if (prep) {
        DecPrepParams pp{packed, max_rounds, chunks, B, N, K, chunk_len, header_bytes, packed_bytes, ctrl, offs};
        decode_prep_kernel<<<1, 1024, 0, stream>>>(pp);
        FCAI_CUDA_TRY(cudaGetLastError());
    }

    DecParams p;
    p.packed = packed;
    p.header_bytes = header_bytes;
    p.max_rounds = max_rounds;
    p.idx = indexes;
    p.medians = medians;
    p.y_out = y_out;
    p.t = TableArgs{cdfs, cdf_sizes, offsets, C, L};
    p.B = B;
    p.N = N;
    p.K = K;
    p.chunk_len = chunk_len;
    p.HW = N / C;
    p.chunks = chunks;
    p.ctrl = ctrl;
    p.offsets = prep ? offs : nullptr;
    p.out = symbols_out;
    const int HW = N / C;
    const int Pg = chunk_len / HW;
    const bool lanes = chunk_len % HW == 0 && lanes_smem(Pg, L, false).bytes <= kMaxSmemBytes;
    if (mode == kModeIdx && !lanes) {
        const int64_t smem = decode_smem_bytes(C, L);
        rc = smem <= kMaxSmemBytes ? launch_decode_full<kModeIdx, true>(p, smem, stream)
                                   : launch_decode_full<kModeIdx, false>(p, smem, stream);
    } else if (chunk_len % HW != 0) {
        const int64_t smem = decode_smem_bytes(C, L);
        const bool sm = smem <= kMaxSmemBytes;
        if (mode == kModeChannel)
            rc = sm ? launch_decode_full<kModeChannel, true>(p, smem, stream)
                    : launch_decode_full<kModeChannel, false>(p, smem, stream);
        else
            rc = sm ? launch_decode_full<kModeLatent, true>(p, smem, stream)
                    : launch_decode_full<kModeLatent, false>(p, smem, stream);
    } else {
        // buckets of at most 64 slots (P <= 8) resolve two-symbol buckets
        // without a search; coarser ones keep the bucket's last symbol
        const int64_t smem = lanes_smem(Pg, L, false).bytes;
        const bool pair = lanes_lut_shift(Pg) <= 6;
        if (lanes) {
            if (mode == kModeIdx)
                rc = pair ? launch_decode_lanes<kModeIdx, true>(p, smem, stream)
                          : launch_decode_lanes<kModeIdx, false>(p, smem, stream);
            else if (mode == kModeChannel)
                rc = pair ? launch_decode_lanes<kModeChannel, true>(p, smem, stream)
                          : launch_decode_lanes<kModeChannel, false>(p, smem, stream);
            else
                rc = pair ? launch_decode_lanes<kModeLatent, true>(p, smem, stream)
                          : launch_decode_lanes<kModeLatent, false>(p, smem, stream);
        }
        else
            rc = mode == kModeChannel ? launch_decode_group<kModeChannel>(p, stream)
                                      : launch_decode_group<kModeLatent>(p, stream);
    }
    if (rc) return rc;
    if (!check) return FCAI_OK;
    long long flags = 0;
    if ((rc = read_status(&ctrl->status[kStFlags], 1, stream, &flags))) return rc;
    if (index_layout_is_channel) *index_layout_is_channel = (flags & kFlagNonChannel) ? 0 : 1;
    return flags_to_status(flags, false);
}

}  // namespace wd

using namespace wd;

extern "C" {

const char *fcai_last_error(void) { return fcai::g_last_error.c_str(); }

const char *fcai_version(void) { return "fcai-b200 0.1.0 (sm_100a)"; }

int fcai_warp_div_plan_create(int32_t B, int32_t N, int32_t C, int32_t P, fcai_warp_div_plan *plan) {
    fcai::clear_error();
    if (!plan) return fcai::fail(FCAI_ERR_INVALID, "plan is null");
    Dims d;
    int rc = make_dims(B, N, C, P, d);
    if (rc) return rc;
    EncLayout el = enc_layout(d.chunks);
    DecLayout dl = dec_layout(d.chunks);
    plan->chunks = d.K;
    plan->chunk_len = d.chunk_len;
    plan->header_bytes = d.header_bytes;
    plan->encode_workspace_bytes = el.fixed_bytes + d.chunks * rows_worst(d) * kLanes * 4;
    plan->decode_workspace_bytes = dl.fixed_bytes;
    plan->max_packed_bytes = d.header_bytes + d.chunks * rows_worst(d) * kLanes * 4;
    return FCAI_OK;
}

int fcai_warp_div_encode(const int32_t *symbols, const int32_t *indexes, int32_t B, int32_t N, const int32_t *cdfs,
                         int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets, int32_t P,
                         void *workspace, int64_t workspace_bytes, uint32_t *max_rounds,
                         fcai_warp_div_encode_info *info, fcai_stream_t stream) {
    fcai::clear_error();
    return encode_impl(indexes ? kModeIdx : kModeChannel, symbols, indexes, nullptr, nullptr, B, N, cdfs, C, L,
                       cdf_sizes, offsets, P, workspace, workspace_bytes, max_rounds, info,
                       reinterpret_cast<cudaStream_t>(stream));
}

int fcai_warp_div_encode_latent(const float *y, const float *medians, int32_t B, int32_t N, const int32_t *cdfs,
                                int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets, int32_t P,
                                void *workspace, int64_t workspace_bytes, uint32_t *max_rounds,
                                fcai_warp_div_encode_info *info, fcai_stream_t stream) {
    fcai::clear_error();
    return encode_impl(kModeLatent, nullptr, nullptr, y, medians, B, N, cdfs, C, L, cdf_sizes, offsets, P, workspace,
                       workspace_bytes, max_rounds, info, reinterpret_cast<cudaStream_t>(stream));
}

int fcai_warp_div_encode_latent_submit(const float *y, const float *medians, int32_t B, int32_t N,
                                       const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                                       const int32_t *offsets, int32_t P, void *workspace, int64_t workspace_bytes,
                                       uint32_t *max_rounds, fcai_stream_t stream) {
    fcai::clear_error();
    return encode_impl(kModeLatent, nullptr, nullptr, y, medians, B, N, cdfs, C, L, cdf_sizes, offsets, P, workspace,
                       workspace_bytes, max_rounds, nullptr, reinterpret_cast<cudaStream_t>(stream),
                       StatusPath::kSubmit);
}

int fcai_warp_div_encode_finish(int32_t B, int32_t N, int32_t C, int32_t P, int64_t workspace_bytes,
                                fcai_warp_div_encode_info *info, fcai_stream_t stream_) {
    fcai::clear_error();
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    Dims d;
    int rc = make_dims(B, N, C, P, d);
    if (rc) return rc;
    if (!info) return fcai::fail(FCAI_ERR_INVALID, "null argument");
    MappedStatus ms{};
    if ((rc = mapped_status(stream, &ms))) return rc;
    if (!*ms.pending) return fcai::fail(FCAI_ERR_INVALID, "no encode was submitted on this stream");
    *ms.pending = 0;
    // the submitted encode's status words, not the work enqueued after them
    FCAI_CUDA_TRY(cudaEventSynchronize(ms.done));
    long long status[8];
    for (int i = 0; i < 8; ++i) status[i] = ms.host[8 + i];
    return encode_info_from_status(d, enc_layout(d.chunks), status, workspace_bytes, info);
}

int fcai_warp_div_encode_pack(const void *workspace, int64_t workspace_bytes, int32_t B, int32_t N, int32_t C,
                              int32_t P, uint8_t *packed, int64_t packed_bytes, fcai_stream_t stream_) {
    fcai::clear_error();
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    Dims d;
    int rc = make_dims(B, N, C, P, d);
    if (rc) return rc;
    if (!workspace || !packed) return fcai::fail(FCAI_ERR_INVALID, "null argument");
    EncLayout el = enc_layout(d.chunks);
    if (workspace_bytes < el.fixed_bytes) return fcai::fail(FCAI_ERR_WORKSPACE, "encode workspace too small");
    if (packed_bytes < d.header_bytes || (packed_bytes - d.header_bytes) % (kLanes * 4))
        return fcai::fail(FCAI_ERR_INVALID, "packed size %lld is not a warp_div payload size", (long long)packed_bytes);
    const uint8_t *ws = static_cast<const uint8_t *>(workspace);
    PackParams p;
    p.ctrl = reinterpret_cast<const Control *>(ws);
    p.rounds = reinterpret_cast<const int32_t *>(ws + el.rounds);
    p.used = reinterpret_cast<const int32_t *>(ws + el.used);
    p.offsets = reinterpret_cast<const unsigned long long *>(ws + el.offsets);
    p.stage = reinterpret_cast<const uint32_t *>(ws + el.stage);
    p.chunks = d.chunks;
    p.B = d.B;
    p.N = d.N;
    p.K = d.K;
    p.chunk_len = d.chunk_len;
    p.header_bytes = d.header_bytes;
    p.packed_bytes = packed_bytes;
    p.packed = packed;
    // about 32 warps per SM: several warps share a chunk when chunks are few
    const int64_t target = (int64_t)fcai::sm_count() * 32;
    const int split = (int)std::min<int64_t>(16, std::max<int64_t>(1, target / std::max<int64_t>(d.chunks, 1)));
    const int64_t want = (d.chunks * split + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)fcai::sm_count() * 8;
    const int grid = (int)(want < cap ? want : cap);
    pack_rows_kernel<<<grid, kThreads, 0, stream>>>(p, split);
    FCAI_CUDA_TRY(cudaGetLastError());
    return FCAI_OK;
}

int fcai_warp_div_encode_noalloc(const int32_t *symbols, const int32_t *indexes, int32_t B, int32_t N,
                                 const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                                 const int32_t *offsets, int32_t P, uint8_t *packed, int64_t packed_capacity,
                                 uint32_t *max_rounds, fcai_warp_div_encode_info *info, fcai_stream_t stream_) {
    fcai::clear_error();
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    Dims d;
    int rc = make_dims(B, N, C, P, d);
    if (rc) return rc;
    if (!packed || !info) return fcai::fail(FCAI_ERR_INVALID, "null argument");
    // The worst-case workspace, so the staging can never overflow.
    const int64_t need = enc_layout(d.chunks).fixed_bytes + d.chunks * rows_worst(d) * kLanes * 4;
    if (need > kScratchBytes) {
        info->required_workspace_bytes = need;
        return fcai::fail(FCAI_ERR_WORKSPACE,
                          "encode of %d x %d symbols (P_ch=%d) needs %lld workspace bytes, more than the %lld-byte "
                          "static scratch of fcai_warp_div_encode_noalloc",
                          (int)B, (int)N, (int)P, (long long)need, (long long)kScratchBytes);
    }
    void *scratch = nullptr;
    if ((rc = encode_scratch(&scratch))) return rc;
    // The array keeps the previous call's contents; the control block must
    // start at zero (a call that stopped early may have left it set).
    FCAI_CUDA_TRY(cudaMemsetAsync(scratch, 0, kCtrlBytes, stream));
    // Status words come back by a plain copy into this frame: the mapped
    // pinned slot of the other entry points is created on a stream's first
    // encode (cudaHostAlloc, cudaEventCreate), which this entry point must
    // never do.
    rc = encode_impl(indexes ? kModeIdx : kModeChannel, symbols, indexes, nullptr, nullptr, B, N, cdfs, C, L,
                     cdf_sizes, offsets, P, scratch, need, max_rounds, info, stream, StatusPath::kCopy);
    if (rc) return rc;
    if (info->packed_bytes > packed_capacity)
        return fcai::fail(FCAI_ERR_INVALID, "packed buffer of %lld bytes cannot hold the %lld-byte payload",
                          (long long)packed_capacity, (long long)info->packed_bytes);
    return fcai_warp_div_encode_pack(scratch, need, B, N, C, P, packed, info->packed_bytes, stream_);
}

int fcai_warp_div_decode(const uint8_t *packed, int64_t packed_bytes, const uint32_t *max_rounds, int32_t K,
                         int64_t header_bytes, int32_t chunk_len, const int32_t *indexes, int32_t B, int32_t N,
                         const int32_t *cdfs, int32_t C, int32_t L, const int32_t *cdf_sizes,
                         const int32_t *offsets, int32_t *symbols_out, void *workspace, int64_t workspace_bytes,
                         int32_t check, int32_t *index_layout_is_channel, fcai_stream_t stream) {
    fcai::clear_error();
    return decode_impl(indexes ? kModeIdx : kModeChannel, packed, packed_bytes, max_rounds, K, header_bytes, chunk_len,
                       indexes, B, N, cdfs, C, L, cdf_sizes, offsets, nullptr, symbols_out, nullptr, workspace,
                       workspace_bytes, check, index_layout_is_channel, reinterpret_cast<cudaStream_t>(stream));
}

int fcai_warp_div_decode_latent(const uint8_t *packed, int64_t packed_bytes, const uint32_t *max_rounds, int32_t K,
                                int64_t header_bytes, int32_t chunk_len, int32_t B, int32_t N, const int32_t *cdfs,
                                int32_t C, int32_t L, const int32_t *cdf_sizes, const int32_t *offsets,
                                const float *medians, float *y_hat_out, void *workspace, int64_t workspace_bytes,
                                int32_t check, fcai_stream_t stream) {
    fcai::clear_error();
    return decode_impl(kModeLatent, packed, packed_bytes, max_rounds, K, header_bytes, chunk_len, nullptr, B, N, cdfs,
                       C, L, cdf_sizes, offsets, medians, nullptr, y_hat_out, workspace, workspace_bytes, check,
                       nullptr, reinterpret_cast<cudaStream_t>(stream));
}

int fcai_payload_copy_async(void *dst, const void *src, int64_t bytes, fcai_stream_t stream_) {
    fcai::clear_error();
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fcai::fail(FCAI_ERR_INVALID, "invalid copy arguments");
    if (bytes == 0) return FCAI_OK;
    int dev = 0;
    FCAI_CUDA_TRY(cudaGetDevice(&dev));
    uint8_t *d = static_cast<uint8_t *>(device_address(dst, dev));
    const uint8_t *s = static_cast<const uint8_t *>(device_address(src, dev));
    if (!d || !s)
        return fcai::fail(FCAI_ERR_INVALID,
                          "copy operands must be memory of the current device or pinned host memory mapped into it");
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    const int threads = 256;
    const bool aligned = ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s)) & 15) == 0;
    const int64_t n16 = aligned ? bytes / 16 : 0;
    if (n16 > 0) {
        const int64_t blocks = std::min<int64_t>((n16 + threads - 1) / threads, 148 * 8);
        copy16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(reinterpret_cast<const uint4 *>(s),
                                                                reinterpret_cast<uint4 *>(d), n16);
        FCAI_CUDA_TRY(cudaGetLastError());
    }
    const int64_t rest = bytes - n16 * 16;
    if (rest > 0) {
        const int64_t blocks = std::min<int64_t>((rest + threads - 1) / threads, 148 * 8);
        copy1_kernel<<<(unsigned)blocks, threads, 0, stream>>>(s + n16 * 16, d + n16 * 16, rest);
        FCAI_CUDA_TRY(cudaGetLastError());
    }
    return FCAI_OK;
}

}  // extern "C"
