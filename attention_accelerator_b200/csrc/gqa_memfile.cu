// gqa_memfile.cu -- the reference's ".mem" transport text, decoded and encoded
// on the GPU (pyfiles/gqa_reference.py:26-46, gen_gqa_wrapper_vectors.py:111-119).
//
// Format: one packed AXIS word per line in hex, element 0 in the rightmost 4
// digits (pack_bf16, :26-28).  A reader (read_mem, :44-46) splits the text into
// lines, skips blank lines and lines whose first non-blank characters are "//",
// drops '_' and requires exactly 4 * elements hex digits per remaining line
// (unpack_bf16, :31-36).
//
// Decode, fast path: text written by write_mem (and most files) has R lines of
// exactly 4*elements hex digits and '\n' (the last '\n' optional).  When the
// byte count fits that shape, mem_regular_kernel stages whole lines of the text
// in shared memory (16-byte loads), converts each element's 4 characters with
// byte-parallel (SWAR) arithmetic and checks that every character is a hex
// digit and every line ends in '\n'.  Any mismatch sets a flag in the
// workspace, and the general path below runs; otherwise its kernels return at
// once.  So the call never waits on the host.
//
// Decode, general path, three kernels over the text in device memory:
//   A  count      each thread owns a 64-byte segment of the text (four 16-byte
//                 loads) and every run of non-separator bytes that STARTS in it
//                 (following the run into later segments when it is longer).
//                 A run is blank, a comment, a data row or malformed; the block
//                 sums its data rows, and the first malformed run's byte offset
//                 goes to the result with an atomic minimum.
//   B  scan       one block turns the per-block row counts into row offsets.
//   C  decode     the same walk as A; each data run's row index is the block's
//                 offset + the rows of the block's earlier threads (a block scan)
//                 + the thread's own earlier rows.  The thread converts its hex
//                 digits left to right: digit k belongs to element
//                 elements-1-k/4 (the line is validated in A), and writes the
//                 row two elements per 32-bit store.
// Encode: one thread per 16 bytes of the output text (one division places the
// chunk, then the bytes follow by counting), written with one 16-byte store.
#include "gqa_b200.h"
#include "gqa_internal.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

namespace gqa {

namespace {

constexpr int kSegBytes = 64;
constexpr int kMemThreads = 256;
constexpr int kBlockBytes = kSegBytes * kMemThreads;  // 16 KB of text per block
constexpr int kScanThreads = 1024;
constexpr int kRegularBytes = 16384;  // text staged per block on the fast path
constexpr int kWsFlagBytes = 16;      // workspace: u32 "irregular" flag, then the per-block row counts

// Byte classes.  Separators end a line as str.splitlines does for ASCII text
// (\n, \r, \r\n, \v, \f, \x1c-\x1e); blanks are what str.strip removes inside
// a line (space, \t, \x1f).
__device__ __forceinline__ bool is_sep(uint32_t c) {
    return c == '\n' || c == '\r' || c == 0x0b || c == 0x0c || (c >= 0x1c && c <= 0x1e);
}
__device__ __forceinline__ bool is_blank(uint32_t c) { return c == ' ' || c == '\t' || c == 0x1f; }
__device__ __forceinline__ int hex_value(uint32_t c) {  // -1 if not a hex digit
    if (c >= '0' && c <= '9') return (int)(c - '0');
    const uint32_t l = c | 0x20u;
    if (l >= 'a' && l <= 'f') return (int)(l - 'a' + 10);
    return -1;
}

// The 64 bytes of segment s as 16 words; bytes past the text read as '\n'.
__device__ __forceinline__ void load_segment(const uint8_t* text, uint64_t n, uint64_t s, uint32_t (&w)[16]) {
    const uint64_t base = s * kSegBytes;
    if (base + kSegBytes <= n) {
        const uint4* p = reinterpret_cast<const uint4*>(text + base);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 x = __ldg(p + i);
            w[4 * i] = x.x;
            w[4 * i + 1] = x.y;
            w[4 * i + 2] = x.z;
            w[4 * i + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            uint32_t v = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint64_t pos = base + 4 * i + b;
                v |= (pos < n ? (uint32_t)__ldg(text + pos) : (uint32_t)'\n') << (8 * b);
            }
            w[i] = v;
        }
    }
}

// State of the run being walked.
struct Run {
    uint64_t start;   // byte offset of its first byte
    int nhex;         // hex digits so far
    uint32_t acc;     // nibbles of the element being assembled
    uint32_t pair;    // the element above it, waiting for its partner (decode)
    bool seen;        // a non-blank byte has been seen
    bool gap;         // blanks after a non-blank byte
    bool slash;       // first non-blank byte was '/'
    bool comment;     // "//" line
    bool bad;         // malformed so far
    int kind;         // after the run ends: 0 blank or comment, 1 data row, 2 malformed
};

__device__ __forceinline__ void run_begin(Run& r, uint64_t pos) {
    r.start = pos;
    r.nhex = 0;
    r.acc = 0;
    r.pair = 0;
    r.seen = r.gap = r.slash = r.comment = r.bad = false;
}

// One non-separator byte.  When decoding, every completed element is stored
// into `out` (null: a row past the caller's buffer): elements are completed
// from the highest index down, two per store.  A malformed line with too many
// digits completes indices below 0, which are not stored.
template <bool kDecode>
__device__ __forceinline__ void run_byte(Run& r, uint32_t c, int elements, uint16_t* out) {
    if (r.comment) return;
    if (is_blank(c)) {
        if (r.seen) r.gap = true;
        return;
    }
    if (!r.seen) {
        r.seen = true;
        if (c == '/') {
            r.slash = true;
            return;
        }
    } else if (r.slash) {  // second non-blank byte of a line that began with '/'
        r.slash = false;
        if (c == '/' && !r.gap) {
            r.comment = true;
            return;
        }
        r.bad = true;
    }
    if (r.gap) r.bad = true;  // blank inside the digits
    if (c == '_') return;
    const int v = hex_value(c);
    if (v < 0) {
        r.bad = true;
        return;
    }
    if constexpr (kDecode) {
        r.acc = (r.acc << 4) | (uint32_t)v;
        if ((r.nhex & 3) == 3) {
            const int e = elements - 1 - (r.nhex >> 2);
            if (out == nullptr || e < 0) {
                // not stored
            } else if ((e & 1) == 1 && (elements & 1) == 0) {
                r.pair = r.acc;  // element e, stored with e - 1
            } else if ((elements & 1) == 0) {
                *reinterpret_cast<uint32_t*>(out + e) = (r.pair << 16) | r.acc;
            } else {
                out[e] = (uint16_t)r.acc;
            }
            r.acc = 0;
        }
    }
    ++r.nhex;
}

__device__ __forceinline__ void run_end(Run& r, int elements) {
    if (!r.seen || r.comment) {
        r.kind = 0;
    } else {
        r.kind = (r.bad || r.slash || r.nhex != 4 * elements) ? 2 : 1;
    }
}

struct MemDecodeArgs {
    const uint8_t* text;
    uint64_t n;
    int elements;
    uint16_t* rows;
    uint64_t max_rows;
    uint64_t* block_rows;  // [blocks]  A: rows per block; B: exclusive offsets
    gqa_mem_result* result;
    const uint32_t* irregular;  // set by the fast path: the general path must run
};

// ---------------------------------------------------------------------------
// Fast path.
// ---------------------------------------------------------------------------
struct MemRegularArgs {
    const uint8_t* text;
    uint64_t n;
    int elements;
    uint64_t n_rows;       // R
    int rows_per_block;    // whole lines staged per block
    uint16_t* rows;
    uint64_t max_rows;
    gqa_mem_result* result;
    uint32_t* irregular;
    bool units8;           // elements % 8 == 0 and rows 16-byte aligned: 8 elements per thread step
};

// Byte-parallel checks on 4 ASCII characters (first one in the low byte).  For
// bytes below 0x80, b >= lo iff b + (0x80 - lo) has bit 7 set, and b <= hi iff
// b + (0x7f - hi) has bit 7 clear; no carry crosses a byte.
__device__ __forceinline__ uint32_t in_range4(uint32_t w, uint32_t lo, uint32_t hi) {
    return (w + 0x80808080u - lo) & ~(w + 0x7f7f7f7fu - hi) & 0x80808080u;
}
// 0x80 in every byte that is a hex digit (bytes >= 0x80 give 0 through `ascii`).
__device__ __forceinline__ uint32_t hex_mask4(uint32_t w) {
    const uint32_t ascii = ~w & 0x80808080u;
    const uint32_t low = w & 0x7f7f7f7fu;
    return ascii & (in_range4(low, 0x30303030u, 0x39393939u) | in_range4(low | 0x20202020u, 0x61616161u, 0x66666666u));
}
// The 4 characters' nibbles, two per byte: byte 0 = c0 c1, byte 2 = c2 c3
// (bytes 1 and 3 hold leftovers that the byte permutes below never select).
__device__ __forceinline__ uint32_t nibbles4(uint32_t w) {
    const uint32_t v = (w & 0x0f0f0f0fu) + ((w >> 6) & 0x01010101u) * 9u;  // one nibble per byte
    return (v << 4) | (v >> 8);
}
// Four characters -> their 16-bit value (c0 is the most significant digit).
__device__ __forceinline__ uint32_t hex4(uint32_t w, bool& ok) {
    ok = hex_mask4(w) == 0x80808080u;
    return __byte_perm(nibbles4(w), 0u, 0x4402u);
}

__global__ void __launch_bounds__(kMemThreads) mem_regular_kernel(const __grid_constant__ MemRegularArgs a) {
    __shared__ __align__(16) uint32_t sm[kRegularBytes / 4 + 8];
    const uint64_t width = 4ull * a.elements + 1;
    const uint64_t r0 = (uint64_t)blockIdx.x * a.rows_per_block;
    const uint64_t r1 = min(a.n_rows, r0 + a.rows_per_block);
    if (blockIdx.x == 0 && threadIdx.x == 0) a.result->rows = a.n_rows;
    // Stage text bytes [r0*width, min(r1*width, n)) from the 16-byte boundary below.
    const uint64_t start = r0 * width, end = min(r1 * width, a.n);
    const uint64_t a0 = start & ~15ull;
    const uint64_t vec_end = end & ~15ull;
    uint8_t* sb = reinterpret_cast<uint8_t*>(sm);
    for (uint64_t off = a0 + 16ull * threadIdx.x; off < vec_end; off += 16ull * kMemThreads)
        *reinterpret_cast<uint4*>(sb + (off - a0)) = __ldg(reinterpret_cast<const uint4*>(a.text + off));
    for (uint64_t off = max(vec_end, a0) + threadIdx.x; off < end; off += kMemThreads) sb[off - a0] = a.text[off];
    __syncthreads();
    bool ok = true;
    if (a.units8) {
        // Thread step: 8 elements e0..e0+7 of one row = 32 characters, elements
        // e0+7 .. e0 in text order; one 16-byte store.
        const int per_row = a.elements / 8;
        const int units = (int)(r1 - r0) * per_row;
        const int step_r = kMemThreads / per_row, step_g = kMemThreads % per_row;
        int r = threadIdx.x / per_row, gi = threadIdx.x % per_row;
        uint32_t valid = 0x80808080u;
        for (int u = threadIdx.x; u < units; u += kMemThreads) {
            const uint64_t row = r0 + r;
            const int e0 = 8 * gi;
            const uint32_t o = (uint32_t)(start - a0 + (uint64_t)r * width + 4u * (a.elements - 8 - e0));
            const uint32_t* src = sm + (o >> 2);
            const uint32_t sh = 8 * (o & 3);
            uint32_t w[8];
            uint32_t prev = src[0];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t next = src[k + 1];
                w[k] = __funnelshift_r(prev, next, sh);  // characters of element e0+7-k
                prev = next;
                valid &= hex_mask4(w[k]);
            }
            if (gi == 0) {  // the line's end: '\n', or the text's end after its last line
                const uint64_t nl = row * width + width - 1;
                if (nl < a.n && sb[o + 32] != '\n') valid = 0;
            }
            uint32_t x[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = nibbles4(w[k]);
            // out word i/2 = value(e0+i) | value(e0+i+1) << 16; value(e0+i) comes from w[7-i]
            uint4 q;
            q.x = __byte_perm(x[7], x[6], 0x4602u);
            q.y = __byte_perm(x[5], x[4], 0x4602u);
            q.z = __byte_perm(x[3], x[2], 0x4602u);
            q.w = __byte_perm(x[1], x[0], 0x4602u);
            if (row < a.max_rows) *reinterpret_cast<uint4*>(a.rows + row * a.elements + e0) = q;
            gi += step_g;
            r += step_r;
            if (gi >= per_row) {
                gi -= per_row;
                ++r;
            }
        }
        ok = valid == 0x80808080u;
    }
    const int count = a.units8 ? 0 : (int)(r1 - r0) * a.elements;
    const int step_r = kMemThreads / a.elements, step_e = kMemThreads % a.elements;
    int r = threadIdx.x / a.elements, e = threadIdx.x % a.elements;
    for (int j = threadIdx.x; j < count; j += kMemThreads) {
        const uint64_t row = r0 + r;
        const uint32_t o = (uint32_t)(start - a0 + (uint64_t)r * width + 4u * (a.elements - 1 - e));
        const uint32_t w = __funnelshift_r(sm[o >> 2], sm[(o >> 2) + 1], 8 * (o & 3));
        bool hex;
        const uint32_t val = hex4(w, hex);
        ok &= hex;
        if (e == 0) {  // the line's end: '\n', or the text's end after its last line
            const uint64_t nl = row * width + width - 1;
            if (nl < a.n) ok &= sb[o + 4] == '\n';
        }
        if (row < a.max_rows) a.rows[row * a.elements + e] = (uint16_t)val;
        e += step_e;
        r += step_r;
        if (e >= a.elements) {
            e -= a.elements;
            ++r;
        }
    }
    if (__syncthreads_or(!ok) && threadIdx.x == 0) atomicOr(a.irregular, 1u);
}


// Walks this thread's segment.  For every run that starts in it, calls
// on_run(kind, start) after the run's last byte (which may lie in a later
// segment); on_run returns the row pointer for the thread's next data run.
template <bool kDecode, typename F>
__device__ __forceinline__ void walk_segment(const MemDecodeArgs& a, uint64_t seg, uint16_t* first_row, F&& on_run) {
    const uint64_t base = seg * kSegBytes;
    if (base >= a.n) return;
    uint32_t w[16];
    load_segment(a.text, a.n, seg, w);
    // Does a run continue into this segment from the previous one?
    bool inside = false;
    if (base > 0) inside = !is_sep(__ldg(a.text + base - 1));
    Run r;
    bool mine = false;  // walking a run that started in this segment
    uint16_t* out = first_row;
    uint64_t cur = seg;
    int i = 0;
    for (;;) {
        const uint32_t c = (w[i >> 2] >> (8 * (i & 3))) & 0xffu;
        const uint64_t pos = cur * kSegBytes + i;
        if (is_sep(c)) {
            if (mine) {
                run_end(r, a.elements);
                out = on_run(r.kind, r.start);
                mine = false;
            }
            inside = false;
            if (cur != seg) return;  // the run that crossed over has ended
        } else {
            if (!inside) {
                inside = true;
                mine = true;
                run_begin(r, pos);
            }
            if (mine) run_byte<kDecode>(r, c, a.elements, out);
        }
        if (++i == kSegBytes) {
            if (!mine) return;  // nothing of ours continues
            ++cur;
            i = 0;
            if (cur * kSegBytes >= a.n) {  // the text ends inside the run
                run_end(r, a.elements);
                on_run(r.kind, r.start);
                return;
            }
            load_segment(a.text, a.n, cur, w);
        }
    }
}

__device__ __forceinline__ uint32_t block_sum(uint32_t v, uint32_t* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    uint32_t t = 0;
    for (int i = 0; i < kMemThreads / 32; ++i) t += sh[i];
    return t;
}

// The general kernels loop over the 16 KB chunks with a bounded grid, so that
// after a successful fast path they cost one small launch each.
__global__ void __launch_bounds__(kMemThreads) mem_count_kernel(const __grid_constant__ MemDecodeArgs a, uint64_t chunks) {
    __shared__ uint32_t sh[kMemThreads / 32];
    if (*a.irregular == 0) return;  // the fast path decoded the text
    for (uint64_t chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x) {
        const uint64_t seg = chunk * kMemThreads + threadIdx.x;
        uint32_t rows = 0;
        uint64_t bad = ~0ull;
        walk_segment<false>(a, seg, nullptr, [&](int kind, uint64_t start) -> uint16_t* {
            if (kind != 0) ++rows;
            if (kind == 2 && start < bad) bad = start;
            return nullptr;
        });
        if (bad != ~0ull)
            atomicMin(reinterpret_cast<unsigned long long*>(&a.result->bad_offset), (unsigned long long)bad);
        const uint32_t total = block_sum(rows, sh);
        if (threadIdx.x == 0) a.block_rows[chunk] = total;
        __syncthreads();  // sh is reused by the next chunk
    }
}

// Exclusive scan of the per-block row counts in one block; writes the total.
__global__ void __launch_bounds__(kScanThreads) mem_scan_kernel(uint64_t* counts, uint64_t blocks, gqa_mem_result* res,
                                                                const uint32_t* irregular) {
    __shared__ uint64_t sh[kScanThreads / 32];
    __shared__ uint64_t carry;
    if (*irregular == 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (uint64_t b0 = 0; b0 < blocks; b0 += kScanThreads) {
        const uint64_t i = b0 + threadIdx.x;
        const uint64_t v = i < blocks ? counts[i] : 0;
        uint64_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) sh[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint64_t s = lane < kScanThreads / 32 ? sh[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            if (lane < kScanThreads / 32) sh[lane] = s;  // inclusive warp totals
        }
        __syncthreads();
        const uint64_t before = carry + (warp ? sh[warp - 1] : 0) + x - v;
        if (i < blocks) counts[i] = before;
        __syncthreads();
        if (threadIdx.x == kScanThreads - 1) carry = before + v;
        __syncthreads();
    }
    if (threadIdx.x == 0) res->rows = carry;
}

__device__ __forceinline__ void decode_chunk(const MemDecodeArgs& a, uint64_t chunk, uint32_t* sh) {
    const uint64_t seg = chunk * kMemThreads + threadIdx.x;
    // Rows of this thread's runs (counted again: the walk is cheap next to a
    // scratch array of per-thread counts).
    uint32_t mine = 0;
    walk_segment<false>(a, seg, nullptr, [&](int kind, uint64_t) -> uint16_t* {
        if (kind != 0) ++mine;
        return nullptr;
    });
    // Exclusive scan over the block's threads.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    uint32_t before = x - mine;
    for (int i = 0; i < warp; ++i) before += sh[i];
    if (mine == 0) return;
    uint64_t row = a.block_rows[chunk] + before;
    auto row_ptr = [&](uint64_t r) -> uint16_t* {  // null past the caller's rows
        return r < a.max_rows ? a.rows + r * (uint64_t)a.elements : nullptr;
    };
    walk_segment<true>(a, seg, row_ptr(row), [&](int kind, uint64_t) -> uint16_t* {
        if (kind != 0) ++row;
        return row_ptr(row);
    });
}

__global__ void __launch_bounds__(kMemThreads) mem_decode_kernel(const __grid_constant__ MemDecodeArgs a, uint64_t chunks) {
    __shared__ uint32_t sh[kMemThreads / 32];
    if (*a.irregular == 0) return;
    for (uint64_t chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x) {
        decode_chunk(a, chunk, sh);
        __syncthreads();  // sh is reused by the next chunk
    }
}

struct MemEncodeArgs {
    const uint16_t* rows;
    uint64_t n_rows;
    int elements;
    uint8_t* text;
    uint64_t n;  // text bytes = n_rows * (4 * elements + 1)
};

// Encode: thread per 16 bytes of text.  One division places the chunk's first
// byte at (line, col); the walk then advances col and wraps at the line end.
__global__ void __launch_bounds__(kMemThreads) mem_encode_kernel(const __grid_constant__ MemEncodeArgs a) {
    const uint32_t width = 4u * a.elements + 1;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t ci = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; ci * 16 < a.n; ci += stride) {
        const uint64_t pos = ci * 16;
        uint64_t line = pos / width;
        uint32_t col = (uint32_t)(pos - line * width);
        uint32_t out[4] = {0u, 0u, 0u, 0u};
        uint32_t v = 0;
        const int nb = a.n - pos < 16 ? (int)(a.n - pos) : 16;
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            uint32_t c = 0;
            if (b < nb) {
                if (col == width - 1) {
                    c = '\n';
                } else {
                    if ((col & 3) == 0 || b == 0) v = a.rows[line * a.elements + (a.elements - 1 - (col >> 2))];
                    const uint32_t nib = (v >> (12 - 4 * (col & 3))) & 0xfu;
                    c = nib + (nib < 10 ? '0' : 'a' - 10);
                }
                if (++col == width) {
                    col = 0;
                    ++line;
                }
            }
            out[b >> 2] |= c << (8 * (b & 3));
        }
        if (nb == 16) {
            *reinterpret_cast<uint4*>(a.text + pos) = make_uint4(out[0], out[1], out[2], out[3]);
        } else {
#pragma unroll
            for (int b = 0; b < 16; ++b)
                if (b < nb) a.text[pos + b] = (uint8_t)(out[b >> 2] >> (8 * (b & 3)));
        }
    }
}

uint64_t decode_blocks(size_t text_bytes) { return (text_bytes + kBlockBytes - 1) / kBlockBytes; }

}  // namespace

}  // namespace gqa

extern "C" {

size_t gqa_mem_decode_workspace_bytes(size_t text_bytes) {
    return (size_t)gqa::decode_blocks(text_bytes) * sizeof(uint64_t) + gqa::kWsFlagBytes;
}

int gqa_mem_decode(const void* text, size_t text_bytes, int elements, void* rows, uint64_t max_rows,
                   gqa_mem_result* result, void* workspace, size_t workspace_bytes, void* stream) {
    if (!result || (text_bytes && !text) || (max_rows && !rows)) return GQA_ERR_NULL_POINTER;
    if (elements < 1 || elements > GQA_MEM_MAX_ELEMENTS) return GQA_ERR_GEOMETRY;
    if ((reinterpret_cast<uintptr_t>(text) & 15u) || (reinterpret_cast<uintptr_t>(rows) & 3u))
        return GQA_ERR_ALIGNMENT;
    const uint64_t blocks = gqa::decode_blocks(text_bytes);
    if (blocks && (!workspace || workspace_bytes < gqa_mem_decode_workspace_bytes(text_bytes)))
        return GQA_ERR_WORKSPACE;
    if (blocks > 0x7fffffffull) return GQA_ERR_BATCH;
    const int st = gqa::check_device_memory({text, rows, result, blocks ? workspace : nullptr});
    if (st != GQA_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(result, 0, sizeof(gqa_mem_result), s) != cudaSuccess ||
        cudaMemsetAsync(&result->bad_offset, 0xff, sizeof(result->bad_offset), s) != cudaSuccess)
        return GQA_ERR_CUDA;
    if (!blocks) return GQA_OK;
    uint32_t* irregular = static_cast<uint32_t*>(workspace);
    // The fast path applies when the length is R lines of 4*elements digits + '\n'
    // (the final '\n' optional) and a line fits the staging buffer.
    const uint64_t width = 4ull * elements + 1;
    uint64_t n_rows = 0;
    if (text_bytes % width == 0) n_rows = text_bytes / width;
    else if ((text_bytes + 1) % width == 0) n_rows = (text_bytes + 1) / width;
    const int rows_per_block = (int)((gqa::kRegularBytes - 16) / width);
    const bool regular = n_rows > 0 && rows_per_block >= 1;
    if (cudaMemsetAsync(irregular, regular ? 0 : 1, sizeof(uint32_t), s) != cudaSuccess) return GQA_ERR_CUDA;
    if (regular) {
        gqa::MemRegularArgs f;
        f.text = static_cast<const uint8_t*>(text);
        f.n = text_bytes;
        f.elements = elements;
        f.n_rows = n_rows;
        f.rows_per_block = rows_per_block;
        f.rows = static_cast<uint16_t*>(rows);
        f.max_rows = max_rows;
        f.result = result;
        f.irregular = irregular;
        f.units8 = (elements % 8 == 0) && (reinterpret_cast<uintptr_t>(rows) % 16 == 0);
        const uint64_t fb = (n_rows + rows_per_block - 1) / rows_per_block;
        if (fb > 0x7fffffffull) return GQA_ERR_BATCH;
        gqa::mem_regular_kernel<<<(unsigned)fb, gqa::kMemThreads, 0, s>>>(f);
    }
    gqa::MemDecodeArgs a;
    a.text = static_cast<const uint8_t*>(text);
    a.n = text_bytes;
    a.elements = elements;
    a.rows = static_cast<uint16_t*>(rows);
    a.max_rows = max_rows;
    a.block_rows = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(workspace) + gqa::kWsFlagBytes);
    a.result = result;
    a.irregular = irregular;
    const unsigned grid = (unsigned)std::min<uint64_t>(blocks, 148ull * 8);
    gqa::mem_count_kernel<<<grid, gqa::kMemThreads, 0, s>>>(a, blocks);
    gqa::mem_scan_kernel<<<1, gqa::kScanThreads, 0, s>>>(a.block_rows, blocks, result, irregular);
    gqa::mem_decode_kernel<<<grid, gqa::kMemThreads, 0, s>>>(a, blocks);
    return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

size_t gqa_mem_encode_bytes(uint64_t n_rows, int elements) {
    if (elements < 1 || elements > GQA_MEM_MAX_ELEMENTS) return 0;
    return (size_t)n_rows * (4 * (size_t)elements + 1);
}

int gqa_mem_encode(const void* rows, uint64_t n_rows, int elements, void* text, void* stream) {
    if (elements < 1 || elements > GQA_MEM_MAX_ELEMENTS) return GQA_ERR_GEOMETRY;
    if (!n_rows) return GQA_OK;
    if (!rows || !text) return GQA_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(text) & 15u) || (reinterpret_cast<uintptr_t>(rows) & 1u)) return GQA_ERR_ALIGNMENT;
    const int st = gqa::check_device_memory({rows, text});
    if (st != GQA_OK) return st;
    gqa::MemEncodeArgs a;
    a.rows = static_cast<const uint16_t*>(rows);
    a.n_rows = n_rows;
    a.elements = elements;
    a.text = static_cast<uint8_t*>(text);
    a.n = gqa_mem_encode_bytes(n_rows, elements);
    const uint64_t chunks = (a.n + 15) / 16;
    const unsigned grid = (unsigned)std::min<uint64_t>((chunks + gqa::kMemThreads - 1) / gqa::kMemThreads, 148ull * 16);
    gqa::mem_encode_kernel<<<grid, gqa::kMemThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

}  // extern "C"
