// gqa_chunked.cu -- chunked multi-query GQA decode on the fifth-generation
// tensor cores (tcgen05.mma with TMEM accumulators), sm_100a.
//
// A chunk is up to 128 consecutive query positions t0 .. t0+n-1 of one
// sequence; query i is answered exactly as one single-position call of the
// reference with QUERY_POSITION = t0 + i (gen_gqa_wrapper_vectors.py:121-139):
// RoPE of Q at its position and of every K row at its own, scores scaled by
// 1/sqrt(128) over keys p < SEQ_LEN and p <= t, softmax, weighted V, BF16 RNE.
// With 128 queries per KV head group the work is a dense contraction
// (S = Q K^T, O = P V), so it runs on the tensor cores.
//
// Precision.  The reference rule is <= 64 BF16 ULP against a float64 golden
// with no relative floor: outputs that nearly cancel make it as strict as FP32
// arithmetic.  One BF16 product per operand pair misses it on ~0.5% of the
// outputs, so the rotated Q and K are split into three BF16 parts carrying 24
// significant bits (x = x_h + x_m + x_l) and the products at least 2^-24 of
// the leading one are accumulated in FP32 by the tensor core.  The three K
// parts are stacked as one 192-row B operand, so one k-step of S is three MMAs
// writing three 48-column blocks of TMEM:
//   Q_h [K_h; K_m; K_l]  -> [hh | hm | hl]
//   Q_m [K_h; K_m]       ->      [+mh | +mm]
//   Q_l K_h              ->             [+lh]
// and the softmax reads S = (block 2 + block 1) + block 0.  P in [0, 1] is
// split into three BF16 parts too, and V is exact in BF16.
// The tensor-core accumulator is only trusted over short chains: each 48-key
// tile's P V goes to a fresh TMEM accumulator (9 MMAs), and the softmax threads
// fold it into the running output with correctly rounded FP32 FMAs
// (O = O * 2^(m_old - m_new) + O_tile), which also makes the online-softmax
// rescale exact.
//
// One CTA per (sequence, Q head) unit: M = 128 query rows (TMEM lanes).  The
// units of the last, partly filled wave are split along the keys (a CTA then
// takes a range of tiles and writes FP32 partial rows that chunk_combine_kernel
// merges), so that the wave is filled.
//   warps 0-3   softmax: thread r owns query row r.  Prologue: Q row r rotated
//               at its position, scaled by scale*log2(e), split, stored to
//               shared memory (A operand of S).  Per 48-key tile: S row from
//               TMEM, mask, online softmax, P split into TMEM (A operand of
//               O_tile), and the previous tile's O_tile folded into the running
//               O in TMEM.  Epilogue: O / l -> BF16 row.
//   warps 4-7   K rotation: each 48-key K tile lands (TMA, 128-byte swizzle) in
//               rows 0-47 of its stage; the warps rotate it at the key
//               positions and write the three parts to rows 0-47 / 48-95 /
//               96-143 (B operand of S).
//   warp 8      TMA producer (2-stage rings of K and V tiles), TMEM allocator.
//   warp 9      S issuer and warp 10 P.V issuer (one thread each).
//               tcgen05.mma costs about 65 SM cycles of the issuing thread
//               whatever its size, so every instruction is as large as TMEM
//               allows (N = 144/96/48 for S, 128 for O) and the two streams
//               come from two threads; the 48-key tile is what fits three S
//               blocks, the tile and running O and three P parts in the 512
//               TMEM columns.
#include "gqa_device.cuh"
#include "gqa_internal.h"

#include <cmath>
#include <cstring>

namespace gqa {

namespace {

constexpr int kRows = 128;                      // query rows per CTA
constexpr int kTile = 48;                       // keys per pipeline tile
constexpr int kStages = 2;                      // K and V rings
constexpr int kRowB = 128;                      // one 128-byte swizzle row: 64 BF16
constexpr int kQBlockBytes = kRows * kRowB;     // 128 query rows x 64 dims
constexpr int kQPartBytes = 2 * kQBlockBytes;   // dims 0-63 block, dims 64-127 block
constexpr int kKRows = 3 * kTile;               // K_h, K_m, K_l stacked: 144 rows
constexpr int kKBlockBytes = kKRows * kRowB;    // 144 rows x 64 dims
constexpr int kKStageBytes = 2 * kKBlockBytes;  // two dim blocks
constexpr int kVBlockBytes = kTile * kRowB;     // 48 keys x 64 dims
static_assert(kTile % 16 == 0 && kKBlockBytes % 1024 == 0 && kVBlockBytes % 1024 == 0,
              "whole 16-key MMA steps; 128-byte swizzle atoms stay 1024-byte aligned");
constexpr int kVStageBytes = 2 * kVBlockBytes;
constexpr int kSoftmaxWarps = 4;
constexpr int kRotWarps = 4;
constexpr int kProducerWarp = kSoftmaxWarps + kRotWarps;  // 8
constexpr int kMmaWarp = kProducerWarp + 1;               // 9: issues S = Q K^T
constexpr int kMmaPvWarp = kMmaWarp + 1;                  // 10: issues O_tile = P V
constexpr int kThreads = (kMmaPvWarp + 1) * 32;           // 352
constexpr int kRotThreads = kRotWarps * 32;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;

// TMEM columns (32-bit, 128 lanes): the three S blocks, the tile accumulator
// O_tile, the running O, and the three P parts (A operand: 48 keys = 24 columns
// of BF16 pairs each); every region starts on a 32-column boundary.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;             // 3 x 48 columns
constexpr uint32_t kColOT = 160;
constexpr uint32_t kColO = kColOT + 128;  // 288
constexpr uint32_t kColP = kColO + 128;   // 416
constexpr uint32_t kPStride = 32;         // one P part per 32 columns (24 used)
static_assert(kColS + 3 * kTile <= kColOT && kColP + 2 * kPStride + kTile / 2 <= kTmemCols, "TMEM budget");

// Shared memory: Q parts, K ring, V ring, then barriers and the TMEM base.
constexpr int kOffK = 3 * kQPartBytes;
constexpr int kOffV = kOffK + kStages * kKStageBytes;
constexpr int kOffBars = kOffV + kStages * kVStageBytes;
constexpr int kNumBars = 5 * kStages + 5;
constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;  // + slack to align to 1024 B
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Instruction descriptors (kind::f16): BF16 A and B, FP32 accumulator, M = 128.
//   bits 4-5 D format (1 = F32), 7-9 A format (1 = BF16), 10-12 B format,
//   15 A major (0 = K), 16 B major (1 = MN), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(int n, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kRows >> 4) << 24);
}
constexpr uint32_t kIdescS192 = make_idesc(3 * kTile, false);  // Q_h [K_h; K_m; K_l]^T
constexpr uint32_t kIdescS128 = make_idesc(2 * kTile, false);  // Q_m [K_h; K_m]^T
constexpr uint32_t kIdescS64 = make_idesc(kTile, false);       // Q_l K_h^T
constexpr uint32_t kIdescO = make_idesc(128, true);            // O_tile[128 x 128] (+)= P[128 x 48] V[48 x 128]

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1:
// start >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride byte
// offset >> 4 in 32-45.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

struct alignas(64) ChunkArgs {
    CUtensorMap kmap;   // 4-D (dim, head, row, batch) or (dim, row, head, batch); box 64 dims x 64 rows
    CUtensorMap vmap;
    int kv_rows_inner;  // 1: rows are map dimension 1 (head-major), 0: dimension 2
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    int64_t q_bstride, q_istride, q_hstride;
    int64_t o_bstride, o_istride, o_hstride;
    int seq_len;
    int first_pos;
    int n_queries;
    int n_tiles;       // tiles of a whole (sequence, Q head) unit
    float qscale;
    uint32_t* status;
    const RopeTable* rope;
    // Work split (grid is 1-D): CTAs [0, full_units) each take a whole unit
    // (unit = b * 32 + qh) and write BF16 rows; every later unit is cut into
    // `split` parts of consecutive tiles whose FP32 partial rows go to
    // `partials` ([split unit][part][kRows][132]) for chunk_combine_kernel.
    int full_units;
    int split;
    float* partials;
};

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, one CTA.
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

#define GQA_R32(r)                                                                                                 \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),      \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),      \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),     \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define GQA_W32(r)                                                                                                 \
    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),    \
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),  \
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),  \
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive columns of this thread's TMEM lane (warp w reads lanes 32(w%4)..).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : GQA_R32(r)
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        GQA_W32(r)
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Three BF16 parts of an FP32 pair (element a in the low half): x = h + m + l
// with |x - h - m - l| <= 2^-24 |x| (each residual is exact in FP32).
__device__ __forceinline__ void split3(float a, float b, uint32_t& h, uint32_t& m, uint32_t& l) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(hh);
    const float ra = a - hf.x, rb = b - hf.y;
    const __nv_bfloat162 mm = __floats2bfloat162_rn(ra, rb);
    const float2 mf = __bfloat1622float2(mm);
    h = bf16x2_bits(hh);
    m = bf16x2_bits(mm);
    l = bf16x2_bits(__floats2bfloat162_rn(ra - mf.x, rb - mf.y));
}

// Bounded wait with one outcome for the whole warp, so that the warp-wide
// tcgen05.ld / tcgen05.st that follow are never reached by part of it.
// Three BF16 parts of an FP32 pair with one conversion: the first two parts
// truncate (mask the low 16 bits, so each residual is exact in FP32), the last
// rounds to nearest even: |x - h - m - l| <= 2^-22 |x|.  Fewer F2F conversions
// than split3 for the per-tile operands (P and K).
__device__ __forceinline__ void split3_fast(float a, float b, uint32_t& h, uint32_t& m, uint32_t& l) {
    const uint32_t ha = __float_as_uint(a) & 0xFFFF0000u, hb = __float_as_uint(b) & 0xFFFF0000u;
    h = __byte_perm(ha, hb, 0x7632);
    const float ra = a - __uint_as_float(ha), rb = b - __uint_as_float(hb);
    const uint32_t ma = __float_as_uint(ra) & 0xFFFF0000u, mb = __float_as_uint(rb) & 0xFFFF0000u;
    m = __byte_perm(ma, mb, 0x7632);
    l = bf16x2_bits(__floats2bfloat162_rn(ra - __uint_as_float(ma), rb - __uint_as_float(mb)));
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__device__ __forceinline__ void report_timeout(const ChunkArgs& a) {
    if (a.status) atomicOr(a.status, kDevStatusTimeout);
}


// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA.
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// ---- the kernel -------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) chunked_kernel(const __grid_constant__ ChunkArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // 128-byte swizzle atoms
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* kfull = bars;                 // K tile landed         (tx count)
    uint64_t* krot = kfull + kStages;       // K parts written       (128 rotation threads)
    uint64_t* kempty = krot + kStages;      // S MMAs done with K    (commit)
    uint64_t* vfull = kempty + kStages;     // V tile landed         (tx count)
    uint64_t* vempty = vfull + kStages;     // O_tile MMAs done with V (commit)
    uint64_t* s_full = vempty + kStages;    // S(j) in TMEM          (commit)
    uint64_t* s_free = s_full + 1;          // S(j) read             (128 softmax threads)
    uint64_t* p_full = s_full + 2;          // P(j) in TMEM, O_tile(j-1) read (128 softmax threads)
    uint64_t* pv_done = s_full + 3;         // O_tile(j) complete    (commit)
    uint64_t* q_ready = s_full + 4;         // Q parts in smem       (128 softmax threads)
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
    uint8_t* q_parts = smem;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Which unit (sequence, Q head) and which of its key tiles this CTA takes.
    const int cta = blockIdx.x;
    const bool partial = cta >= a.full_units;
    const int part = partial ? (cta - a.full_units) % a.split : 0;
    const int unit = partial ? a.full_units + (cta - a.full_units) / a.split : cta;
    const int nparts = partial ? a.split : 1;
    const int j0 = (int)((int64_t)a.n_tiles * part / nparts);
    const int j1 = (int)((int64_t)a.n_tiles * (part + 1) / nparts);
    const int qh = unit % kNumQHeads;  // Q head
    const int kvh = qh / kGroup;       // its KV head
    const int b = unit / kNumQHeads;   // sequence
    const RopeTable* rt = a.rope;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kfull[s], 1);
            mbar_init(&krot[s], kRotThreads);
            mbar_init(&kempty[s], 1);
            mbar_init(&vfull[s], 1);
            mbar_init(&vempty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kSoftmaxThreads);
        mbar_init(p_full, kSoftmaxThreads);
        mbar_init(pv_done, 1);
        mbar_init(q_ready, kSoftmaxThreads);
        fence_barrier_init();
    }
    if (warp == kProducerWarp) {  // whole warp: TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(tmem_base_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        if (lane == 0) {
            prefetch_tensormap(&a.kmap);
            prefetch_tensormap(&a.vmap);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_slot;
    const int n_tiles = j1 - j0;  // this CTA's tiles: absolute tiles j0 .. j1-1

    if (warp < kSoftmaxWarps) {
        // ======================= softmax: thread r owns query row r =======================
        const int r = threadIdx.x;                       // TMEM lane r (warp w: lanes 32w..32w+31)
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const bool row_ok = r < a.n_queries;
        const int qpos = a.first_pos + r;
        const int last_key = row_ok ? min(a.seq_len - 1, qpos) : -1;  // keys 0..last_key are visible
        bool ok = true;

        // Q row rotated at its position, scaled, split into three parts: row r of
        // each part's two 128-byte-swizzled dim blocks (A operand of S).
        {
            const __nv_bfloat16* qrow = a.q + (int64_t)b * a.q_bstride + (int64_t)r * a.q_istride +
                                        (int64_t)qh * a.q_hstride;
            for (int c8 = 0; c8 < 8; ++c8) {  // pairs 8 c8 .. 8 c8 + 7: chunk c8 of both dim blocks
                uint4 xr4 = make_uint4(0u, 0u, 0u, 0u), yr4 = xr4;
                if (row_ok) {
                    xr4 = *reinterpret_cast<const uint4*>(qrow + 8 * c8);
                    yr4 = *reinterpret_cast<const uint4*>(qrow + 64 + 8 * c8);
                }
                const uint32_t xw[4] = {xr4.x, xr4.y, xr4.z, xr4.w};
                const uint32_t yw[4] = {yr4.x, yr4.y, yr4.z, yr4.w};
                uint32_t xp[3][4], yp[3][4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const float2 x = bf16x2_to_float2(xw[w]), y = bf16x2_to_float2(yw[w]);
                    const float2 f0 = rope_factor(rt->step[8 * c8 + 2 * w], qpos);
                    const float2 f1 = rope_factor(rt->step[8 * c8 + 2 * w + 1], qpos);
                    const float x0 = (x.x * f0.x - y.x * f0.y) * a.qscale;
                    const float y0 = (x.x * f0.y + y.x * f0.x) * a.qscale;
                    const float x1 = (x.y * f1.x - y.y * f1.y) * a.qscale;
                    const float y1 = (x.y * f1.y + y.y * f1.x) * a.qscale;
                    split3(x0, x1, xp[0][w], xp[1][w], xp[2][w]);
                    split3(y0, y1, yp[0][w], yp[1][w], yp[2][w]);
                }
                const int off = r * kRowB + ((c8 ^ (r & 7)) << 4);
#pragma unroll
                for (int pi = 0; pi < 3; ++pi) {
                    uint8_t* part = q_parts + pi * kQPartBytes;
                    *reinterpret_cast<uint4*>(part + off) = make_uint4(xp[pi][0], xp[pi][1], xp[pi][2], xp[pi][3]);
                    *reinterpret_cast<uint4*>(part + kQBlockBytes + off) =
                        make_uint4(yp[pi][0], yp[pi][1], yp[pi][2], yp[pi][3]);
                }
            }
            fence_proxy_async_smem();  // the tensor core reads Q through the async proxy
            mbar_arrive(q_ready);
        }

        float m_run = -INFINITY;  // running max of the row (log2 units)
        float l = 0.f;            // running sum of 2^(s - m_run)
        float alpha_prev = 1.f;   // alpha of the tile whose O_tile is folded next
        for (int j = 0; j < n_tiles && ok; ++j) {
            if (!warp_wait(s_full, j & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int k0 = (j0 + j) * kTile;
            // S = (block 2 + block 1) + block 0, in two load batches (one wait each).
            float s[kTile];
            float mx = -INFINITY;
            {
                uint32_t b2[kTile], b1[kTile];
#pragma unroll
                for (int c16 = 0; c16 < kTile / 16; ++c16) {
                    tmem_ld16(lane_base + kColS + 2 * kTile + 16 * c16, *reinterpret_cast<uint32_t(*)[16]>(&b2[16 * c16]));
                    tmem_ld16(lane_base + kColS + kTile + 16 * c16, *reinterpret_cast<uint32_t(*)[16]>(&b1[16 * c16]));
                }
                tmem_wait_ld();
#pragma unroll
                for (int col = 0; col < kTile; ++col) s[col] = __uint_as_float(b2[col]) + __uint_as_float(b1[col]);
            }
            {
                uint32_t b0[kTile];
#pragma unroll
                for (int c16 = 0; c16 < kTile / 16; ++c16)
                    tmem_ld16(lane_base + kColS + 16 * c16, *reinterpret_cast<uint32_t(*)[16]>(&b0[16 * c16]));
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(s_free);
                if (k0 + kTile - 1 <= last_key) {  // every key of the tile is visible to this row
#pragma unroll
                    for (int col = 0; col < kTile; ++col) {
                        s[col] += __uint_as_float(b0[col]);
                        mx = fmaxf(mx, s[col]);
                    }
                } else {
#pragma unroll
                    for (int col = 0; col < kTile; ++col) {
                        const float v = s[col] + __uint_as_float(b0[col]);
                        s[col] = k0 + col <= last_key ? v : -INFINITY;
                        mx = fmaxf(mx, s[col]);
                    }
                }
            }

            const float m_new = fmaxf(m_run, mx);
            const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);  // 0 for the first visible key
            m_run = m_new;
            // A row with no visible key yet (possible in a later part of a split
            // unit) exponentiates against 0: its P stays 0 rather than NaN.
            const float m_use = m_run == -INFINITY ? 0.f : m_run;
            l *= alpha;
            // P(j) = 2^(s - m_run) split into three parts, in registers while O_tile(j-1) may still
            // be in flight (keys 2c, 2c+1 in column c of each part: the A operand of O_tile).
            float psum0 = 0.f, psum1 = 0.f;
            uint32_t pp[3][kTile / 2];
#pragma unroll
            for (int c = 0; c < kTile; c += 2) {
                // ex2(-inf) = 0 for masked keys; rows without any visible key (past
                // n_queries) produce values that are never written out.
                const float p0 = fast_exp2(s[c] - m_use);
                const float p1 = fast_exp2(s[c + 1] - m_use);
                psum0 += p0;
                psum1 += p1;
                split3_fast(p0, p1, pp[0][c >> 1], pp[1][c >> 1], pp[2][c >> 1]);
            }
            const float psum = psum0 + psum1;
            if (j > 0) {
                // O_tile(j-1) is complete and the P columns are free once O_tile(j-1) is done.
                if (!warp_wait(pv_done, (j - 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
#pragma unroll
            for (int pi = 0; pi < 3; ++pi) {
                tmem_st16(lane_base + kColP + kPStride * pi, *reinterpret_cast<const uint32_t(*)[16]>(&pp[pi][0]));
                tmem_st8(lane_base + kColP + kPStride * pi + 16, *reinterpret_cast<const uint32_t(*)[8]>(&pp[pi][16]));
            }
            if (j > 0) {
                // The fold of O_tile(j-1) into the running O, in 32-column chunks:
                //   O(t) = O(t-1) * alpha(t) + O_tile(t),  alpha(t) = 2^(m(t-1) - m(t)).
#pragma unroll 1
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint32_t ot[32], o[32];
                    tmem_ld32(lane_base + kColOT + 32 * q4, ot);
                    if (j > 1) tmem_ld32(lane_base + kColO + 32 * q4, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        o[c] = __float_as_uint(j > 1 ? fmaf(__uint_as_float(o[c]), alpha_prev, __uint_as_float(ot[c]))
                                                     : __uint_as_float(ot[c]));
                    tmem_st32(lane_base + kColO + 32 * q4, o);
                }
            }
            l += psum;
            alpha_prev = alpha;
            tmem_wait_st();
            tc_fence_before();  // P stores and the tcgen05.ld of O_tile(j-1) precede the arrival
            mbar_arrive(p_full);
        }
        if (ok && warp_wait(pv_done, (n_tiles - 1) & 1)) {
            tc_fence_after();
            // O = O(n-2) * alpha + O_tile(n-1), then O / l rounded to BF16, or for a
            // part of a split unit the FP32 partial row (acc, m, l).
            __nv_bfloat16* orow =
                a.out + (int64_t)b * a.o_bstride + (int64_t)r * a.o_istride + (int64_t)qh * a.o_hstride;
            float* prow = partial ? a.partials + ((size_t)(cta - a.full_units) * kRows + r) * kPartialFloats
                                  : nullptr;
            if (partial && row_ok) {
                prow[kHeadDim] = m_run;
                prow[kHeadDim + 1] = l;
            }
#pragma unroll 1
            for (int q4 = 0; q4 < 4; ++q4) {
                uint32_t ot[32], o[32];
                tmem_ld32(lane_base + kColOT + 32 * q4, ot);
                if (n_tiles > 1) tmem_ld32(lane_base + kColO + 32 * q4, o);
                tmem_wait_ld();
                if (row_ok && partial) {
#pragma unroll
                    for (int c = 0; c < 32; c += 4) {
                        float v4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            v4[e] = n_tiles > 1 ? fmaf(__uint_as_float(o[c + e]), alpha_prev, __uint_as_float(ot[c + e]))
                                                : __uint_as_float(ot[c + e]);
                        *reinterpret_cast<float4*>(prow + 32 * q4 + c) = make_float4(v4[0], v4[1], v4[2], v4[3]);
                    }
                } else if (row_ok) {
#pragma unroll
                    for (int c = 0; c < 32; c += 8) {
                        float v8[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float acc = n_tiles > 1 ? fmaf(__uint_as_float(o[c + e]), alpha_prev,
                                                                 __uint_as_float(ot[c + e]))
                                                          : __uint_as_float(ot[c + e]);
                            v8[e] = acc / l;
                        }
                        uint4 w;
                        w.x = bf16x2_bits(__floats2bfloat162_rn(v8[0], v8[1]));
                        w.y = bf16x2_bits(__floats2bfloat162_rn(v8[2], v8[3]));
                        w.z = bf16x2_bits(__floats2bfloat162_rn(v8[4], v8[5]));
                        w.w = bf16x2_bits(__floats2bfloat162_rn(v8[6], v8[7]));
                        *reinterpret_cast<uint4*>(orow + 32 * q4 + c) = w;
                    }
                }
            }
        } else {
            ok = false;
        }
        if (!ok) report_timeout(a);
    } else if (warp < kSoftmaxWarps + kRotWarps) {
        // ======================= K rotation + split =======================
        // Thread t: pairs 8c .. 8c+7 (16-byte chunk c of both dim blocks), keys kq + 16u, u < 3.
        const int t = threadIdx.x - kSoftmaxThreads;
        const int c = t & 7;
        const int kq = t >> 3;
        // Factors of this thread's pairs at its first key of the tile: exact every
        // kReanchorTiles tiles, otherwise the previous tile's times e^{i theta 48}.
        constexpr int kReanchorTiles = 2;
        float2 step16[8], step_tile[8], base[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            step16[i] = rope_factor(rt->step[8 * c + i], 16);
            step_tile[i] = rope_factor(rt->step[8 * c + i], kTile);
        }
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int st = j % kStages;
            if (!mbar_wait(&kfull[st], (j / kStages) & 1)) {
                ok = false;
                break;
            }
            uint8_t* kb = smem + kOffK + st * kKStageBytes;  // dim block 0; block 1 at + kKBlockBytes
            float2 f[8];
            if (j % kReanchorTiles == 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) base[i] = rope_factor(rt->step[8 * c + i], (int64_t)(j0 + j) * kTile + kq);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float2 g = base[i], st1 = step_tile[i];
                    base[i] = make_float2(g.x * st1.x - g.y * st1.y, g.x * st1.y + g.y * st1.x);
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = base[i];
#pragma unroll 1
            for (int u = 0; u < kTile / 16; ++u) {
                const int k = kq + 16 * u;
                const int off = k * kRowB + ((c ^ (k & 7)) << 4);  // 128-byte swizzle: chunk c of row k
                const uint4 xv = *reinterpret_cast<const uint4*>(kb + off);
                const uint4 yv = *reinterpret_cast<const uint4*>(kb + kKBlockBytes + off);
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
                const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
                uint32_t xh[4], xm[4], xl[4], yh[4], ym[4], yl[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const float2 x = bf16x2_to_float2(xw[w]), y = bf16x2_to_float2(yw[w]);
                    const float2 f0 = f[2 * w], f1 = f[2 * w + 1];
                    split3_fast(x.x * f0.x - y.x * f0.y, x.y * f1.x - y.y * f1.y, xh[w], xm[w], xl[w]);
                    split3_fast(x.x * f0.y + y.x * f0.x, x.y * f1.y + y.y * f1.x, yh[w], ym[w], yl[w]);
                }
                // Row k of K_h, row 48 + k of K_m, row 96 + k of K_l (the row swizzle is the same:
                // 48 and 96 are multiples of 8).
                constexpr int kPartRows = kTile * kRowB;
                *reinterpret_cast<uint4*>(kb + off) = make_uint4(xh[0], xh[1], xh[2], xh[3]);
                *reinterpret_cast<uint4*>(kb + kKBlockBytes + off) = make_uint4(yh[0], yh[1], yh[2], yh[3]);
                *reinterpret_cast<uint4*>(kb + kPartRows + off) = make_uint4(xm[0], xm[1], xm[2], xm[3]);
                *reinterpret_cast<uint4*>(kb + kKBlockBytes + kPartRows + off) = make_uint4(ym[0], ym[1], ym[2], ym[3]);
                *reinterpret_cast<uint4*>(kb + 2 * kPartRows + off) = make_uint4(xl[0], xl[1], xl[2], xl[3]);
                *reinterpret_cast<uint4*>(kb + kKBlockBytes + 2 * kPartRows + off) =
                    make_uint4(yl[0], yl[1], yl[2], yl[3]);
                // Factors 16 keys further on.
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float2 g = f[i], sst = step16[i];
                    f[i] = make_float2(g.x * sst.x - g.y * sst.y, g.x * sst.y + g.y * sst.x);
                }
            }
            fence_proxy_async_smem();  // the tensor core reads these parts through the async proxy
            mbar_arrive(&krot[st]);
        }
        if (!ok) report_timeout(a);
    } else if (warp == kProducerWarp) {
        // ======================= TMA producer =======================
        if (lane == 0) {
            bool ok = true;
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int row = (j0 + j) * kTile;
                const int c1 = a.kv_rows_inner ? row : kvh;
                const int c2 = a.kv_rows_inner ? kvh : row;
                const int st = j % kStages;
                if (j >= kStages && !mbar_wait(&kempty[st], ((j / kStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                uint8_t* kb = smem + kOffK + st * kKStageBytes;
                mbar_arrive_expect_tx(&kfull[st], 2 * kVBlockBytes);
                tma_load_4d(kb, &a.kmap, 0, c1, c2, b, &kfull[st]);                 // rows 0-47, dims 0-63
                tma_load_4d(kb + kKBlockBytes, &a.kmap, 64, c1, c2, b, &kfull[st]);  // rows 0-47, dims 64-127
                if (j >= kStages && !mbar_wait(&vempty[st], ((j / kStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                uint8_t* vb = smem + kOffV + st * kVStageBytes;
                mbar_arrive_expect_tx(&vfull[st], kVStageBytes);
                tma_load_4d(vb, &a.vmap, 0, c1, c2, b, &vfull[st]);
                tma_load_4d(vb + kVBlockBytes, &a.vmap, 64, c1, c2, b, &vfull[st]);
            }
            if (!ok) report_timeout(a);
        }
    } else if (warp == kMmaWarp) {
        // ======================= MMA issuer: S =======================
        if (lane == 0) {
            bool ok = mbar_wait(q_ready, 0);
            tc_fence_after();
            const uint32_t t_s = tmem + kColS;
            const uint32_t qh_addr = smem_addr(q_parts);
            // S(j), 16 dims per k-step kk (dim block kk / 4, 32 bytes per step within the row).
            auto issue_s = [&](int j) {
                const uint32_t kaddr = smem_addr(smem + kOffK + (j % kStages) * kKStageBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t koff = (kk >> 2) * kKBlockBytes + (kk & 3) * 32;
                    const uint32_t qoff = (kk >> 2) * kQBlockBytes + (kk & 3) * 32;
                    const uint64_t bd = smem_desc_sw128(kaddr + koff, 16, 1024);
                    mma_ss(t_s, smem_desc_sw128(qh_addr + qoff, 16, 1024), bd, kIdescS192, kk != 0);
                    mma_ss(t_s + kTile, smem_desc_sw128(qh_addr + kQPartBytes + qoff, 16, 1024), bd, kIdescS128, 1u);
                    mma_ss(t_s + 2 * kTile, smem_desc_sw128(qh_addr + 2 * kQPartBytes + qoff, 16, 1024), bd,
                           kIdescS64, 1u);
                }
                tc_commit(s_full);
                tc_commit(&kempty[j % kStages]);
            };
            // S(j) once K(j) is rotated and the softmax has read S(j-1).  The P.V
            // products are issued by the next warp, so the two streams of MMAs
            // overlap their issue.
            for (int j = 0; j < n_tiles && ok; ++j) {
                if (!mbar_wait(&krot[j % kStages], (j / kStages) & 1) || (j > 0 && !mbar_wait(s_free, (j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_s(j);
            }
            if (!ok) report_timeout(a);
        }
    } else if (warp == kMmaPvWarp) {
        // ======================= MMA issuer: P.V =======================
        if (lane == 0) {
            bool ok = true;
            const uint32_t t_ot = tmem + kColOT, t_p = tmem + kColP;
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int st = j % kStages;
                if (!mbar_wait(p_full, j & 1) || !mbar_wait(&vfull[st], (j / kStages) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // O_tile(j) = P_l V + P_m V + P_h V: 16 keys per MMA (16 rows of 128 bytes).
                const uint32_t vaddr = smem_addr(smem + kOffV + st * kVStageBytes);
#pragma unroll
                for (int pi = 2; pi >= 0; --pi) {
#pragma unroll
                    for (int kk = 0; kk < kTile / 16; ++kk) {
                        const uint64_t bd = smem_desc_sw128(vaddr + kk * 16 * kRowB, kVBlockBytes, 1024);
                        mma_ts(t_ot, t_p + kPStride * pi + 8 * kk, bd, kIdescO, (pi != 2 || kk != 0) ? 1u : 0u);
                    }
                }
                tc_commit(pv_done);
                tc_commit(&vempty[st]);
            }
            if (!ok) report_timeout(a);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// LSE merge of a split unit's parts (the reference's flash-softmax rescale,
// flash_softmax.v:233-512, output_accumulator.v:398-687, across key ranges):
// one CTA per (split unit, query row), one thread per dim.
__global__ void __launch_bounds__(kHeadDim) chunk_combine_kernel(const float* __restrict__ partials, int full_units,
                                                                 int split, int n_queries, __nv_bfloat16* out,
                                                                 int64_t o_bstride, int64_t o_istride,
                                                                 int64_t o_hstride) {
    const int su = blockIdx.x / n_queries, r = blockIdx.x % n_queries;
    const int unit = full_units + su;
    const int b = unit / kNumQHeads, qh = unit % kNumQHeads;
    const int d = threadIdx.x;
    auto row = [&](int p) { return partials + ((size_t)(su * split + p) * kRows + r) * kPartialFloats; };
    float M = -INFINITY;
    for (int p = 0; p < split; ++p) M = fmaxf(M, row(p)[kHeadDim]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
    for (int p = 0; p < split; ++p) {
        const float* x = row(p);
        const float f = exp2f(x[kHeadDim] - Mu);
        L = fmaf(x[kHeadDim + 1], f, L);
        O = fmaf(x[d], f, O);
    }
    out[(int64_t)b * o_bstride + (int64_t)r * o_istride + (int64_t)qh * o_hstride + d] = __float2bfloat16_rn(O / L);
}

}  // namespace

void chunked_split_plan(int batch, int seq_len, int first_pos, int n_queries, int sms, int* full_units, int* split) {
    // The units of the last, partly filled wave are cut along the keys so
    // that they fill it: with U units on `sms` SMs the rem = U mod sms units
    // left after the full waves become rem * s CTAs, s = floor(sms / rem),
    // each part at least kMinPartTiles tiles.
    constexpr int kMinPartTiles = 4;
    const int units = batch * kNumQHeads;
    const int n_keys = first_pos + n_queries < seq_len ? first_pos + n_queries : seq_len;
    const int n_tiles = (n_keys + kTile - 1) / kTile;
    const int rem = units % sms;
    int s = rem ? sms / rem : 1;
    if (s > n_tiles / kMinPartTiles) s = n_tiles / kMinPartTiles;
    if (s < 2) {
        *full_units = units;
        *split = 1;
    } else {
        *full_units = units - rem;
        *split = s;
    }
}

size_t chunked_partial_bytes(int batch, int full_units, int split) {
    if (split < 2) return 0;
    return (size_t)(batch * kNumQHeads - full_units) * split * kRows * kPartialFloats * sizeof(float);
}

size_t chunked_smem_bytes() { return kSmemBytes; }
int chunked_max_queries() { return kRows; }
int chunked_tile_keys() { return kTile; }

cudaError_t chunked_prepare() {
    return cudaFuncSetAttribute(chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

cudaError_t launch_chunked(const ChunkLaunch& l, cudaStream_t stream) {
    ChunkArgs a;
    memset(&a, 0, sizeof(a));
    a.kmap = l.kmap;
    a.vmap = l.vmap;
    a.kv_rows_inner = l.kv_rows_inner;
    a.q = static_cast<const __nv_bfloat16*>(l.q);
    a.out = static_cast<__nv_bfloat16*>(l.out);
    a.q_bstride = l.q_bstride;
    a.q_istride = l.q_istride;
    a.q_hstride = l.q_hstride;
    a.o_bstride = l.o_bstride;
    a.o_istride = l.o_istride;
    a.o_hstride = l.o_hstride;
    a.seq_len = l.seq_len;
    a.first_pos = l.first_pos;
    a.n_queries = l.n_queries;
    const int n_keys = l.first_pos + l.n_queries < l.seq_len ? l.first_pos + l.n_queries : l.seq_len;
    a.n_tiles = (n_keys + kTile - 1) / kTile;
    a.qscale = l.qscale;
    a.status = l.status;
    a.rope = l.rope;
    const int units = l.batch * kNumQHeads;
    a.full_units = l.split >= 2 ? l.full_units : units;
    a.split = l.split >= 2 ? l.split : 1;
    a.partials = l.partials;
    const int split_units = units - a.full_units;
    chunked_kernel<<<a.full_units + split_units * a.split, kThreads, kSmemBytes, stream>>>(a);
    if (split_units > 0)
        chunk_combine_kernel<<<split_units * l.n_queries, kHeadDim, 0, stream>>>(
            l.partials, a.full_units, a.split, l.n_queries, static_cast<__nv_bfloat16*>(l.out), l.o_bstride,
            l.o_istride, l.o_hstride);
    return cudaGetLastError();
}

}  // namespace gqa
