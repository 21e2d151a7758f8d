// gqa_decode.cu -- split-KV flash-decoding kernels for GQA (32 Q heads over 8 KV
// heads, head_dim 128) on sm_100a: the decode kernel, the split merge, the
// cross-shard log-sum-exp combine and a stand-alone RoPE kernel.
//
// decode_kernel: one CTA computes the attention of the 4 Q heads of one KV head
// h of one sequence b over a contiguous range of that sequence's visible keys
// (a "split").  This is the reference's per-KV-head group loop
// (gqa_controller.v:140-277: Q group -> K position -> block) with the key loop
// cut into splits so that every SM streams K/V rows at once.
//   warp 11     producer: works out the CTA's (sequence, split), then one thread
//               issues the group's 4 Q rows and, per 88-key tile, one TMA tensor
//               copy for K and one for V (22 KB each, one head, any K/V strides)
//               into a 4-stage shared-memory ring, one mbarrier per stage and
//               direction.  The warp also writes each stage's Q rotated to the
//               tile's first key position (RoPE is relative), so that the
//               consumers rotate K by fixed per-lane factors only.
//   warps 0..10 consumers: warp c owns keys [8c, 8c+8) of every tile, four at a
//               time: 8 lanes per key, each lane 8 rotate_half pairs (16 of the
//               128 dims).  Per key: RoPE of K (rope_unit.v) relative to the
//               tile's first key, the 4 Q.K dot
//               products in FP32 (bf16_dot_product_mac.v + scale_unit.v), a
//               3-level shuffle reduction, online softmax in log2 units
//               (flash_softmax.v:233-490) and the P.V accumulation
//               (output_accumulator.v:244-536) with each lane owning 4 dims.
//               The Q.K and softmax of tile t and the P.V of tile t-1 form
//               one branch-free block, so that they interleave.
//   epilogue    the 11 warps' (m, l, acc) merge through shared memory; a sequence
//               with one split writes its BF16 rows (O * 1/l,
//               output_accumulator.v:546-687) directly.  Otherwise each split
//               writes an FP32 partial: for a batch, split_merge_kernel merges
//               them; for a single sequence the last split of each KV head to
//               finish merges them (arrival counter in the workspace header),
//               and with gqa_decode_exchange also swaps the merged rows with
//               the other GPUs of a sequence split over NVLink peer memory.
//   cluster     (single sequence of up to 16 splits) the splits of one KV head
//               run as one thread-block cluster: each keeps its partial in
//               shared memory and, after a cluster barrier, merges 32 of the
//               head group's 512 outputs from all the cluster's partials over
//               distributed shared memory -- no second kernel, no workspace
//               round trip.
// Both kernels are launched with programmatic dependent launch: everything that
// reads only the argument block (barrier set-up, RoPE tables) runs before
// griddepcontrol.wait, overlapping the tail of the previous kernel in the
// stream; a single sequence's split also prefetches its Q rows and first K/V
// tiles into L2 there.  A batch's CTAs take every sequence's full-chunk splits
// first and the shorter last splits after them, so that those fill the last wave.
#include "gqa_b200.h"
#include "gqa_device.cuh"
#include "gqa_internal.h"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace gqa {

namespace {

// 11 consumer warps + 1 producer warp = 12 warps: the most warps the 157
// registers a consumer thread needs allow (160 allocated; 64K registers per
// SM; at 16 warps the allocation would be 128).
constexpr int kConsumerWarps = kDecodeConsumerWarps;
constexpr int kKeysPerWarp = kDecodeKeysPerWarp;  // keys of one tile per warp
constexpr int kTileKeys = kDecodeTileKeys;        // 88 keys per pipeline tile
constexpr int kStages = 4;
constexpr int kSteps = kKeysPerWarp / 4;                  // groups of 4 keys (8 lanes per key)
static_assert(kSteps >= 1 && kSteps * 4 == kKeysPerWarp, "a warp takes whole groups of 4 keys");
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;  // + the producer warp
constexpr int kTileBytes = kTileKeys * kRowBytes;
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kReanchorTiles = 32;  // exact RoPE phase every 32 tiles (2816 keys)
// Epilogue: consumer thread tid owns outputs o = tid, tid + kConsumerThreads, ...
// of the 4 x 128 (head, dim) outputs.
constexpr int kOutputs = kGroup * kHeadDim;

// Shared-memory layout.
constexpr int kOffBars = kStages * kStageBytes;       // full[kStages], empty[kStages], q
constexpr int kOffQ = kOffBars + (2 * kStages + 2) * 8;  // the group's 4 Q rows (BF16)
constexpr int kOffP = kOffQ + kGroup * kRowBytes;
constexpr int kPBytes = 2 * kConsumerWarps * kKeysPerWarp * kGroup * 4;  // [warp][2][key][head] p
constexpr int kOffAlpha = kOffP + kPBytes;
// Exact RoPE factors of Q at QUERY_POSITION shared by the CTA's lanes (float2,
// kPairs), for a pre-rotated K cache.
constexpr int kRopeQ = 0, kRopeRows = 1;
constexpr int kOffRope = kOffAlpha + 2 * kConsumerWarps * kGroup * 4;
constexpr int kOffInfo = kOffRope + kRopeRows * kPairs * 8;
// Per stage, the group's Q rotated to the tile's first key and pre-scaled
// (FP32, written by the producer warp): [head][re, im][half][g][4], so that
// pair 8g + 4 half + e of a head's re (im) part sits at half*32 + 4g + e and a
// consumer lane's two 16-byte loads per part are contiguous across g.
constexpr int kQtFloats = kGroup * kHeadDim;
constexpr int kOffQt = kOffInfo + 64;
constexpr int kSmemBytes = kOffQt + kStages * kQtFloats * 4;
static_assert(kOffQt % 16 == 0, "16-byte loads of the rotated Q");
static_assert(kConsumerWarps * kGroup * kPartialFloats * 4 <= kOffBars, "warp merge buffer fits the ring");

// Splits per sequence that split_merge_kernel merges in one pass.
constexpr int kMaxSplitsPerSeq = 64;

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Complex multiply of (re, im) pairs held as float2 lanes: (ar + i ai) * (br + i bi).
__device__ __forceinline__ void cmul2(float2 ar, float2 ai, float2 br, float2 bi, float2& cr, float2& ci) {
    const float2 nbi = make_float2(-bi.x, -bi.y);
    cr = __ffma2_rn(ar, br, __fmul2_rn(ai, nbi));
    ci = __ffma2_rn(ar, bi, __fmul2_rn(ai, br));
}

// acc + (p, p) * v with p broadcast to both halves of the packed operand
// (one 16-byte load then serves the 4 heads' probabilities of a key).
__device__ __forceinline__ float2 ffma2_bcast(float p, float2 v, float2 acc) {
    uint64_t r;
    asm("{\n\t.reg .b64 pp;\n\tmov.b64 pp, {%1, %1};\n\tfma.rn.f32x2 %0, pp, %2, %3;\n\t}"
        : "=l"(r)
        : "f"(p), "l"(*reinterpret_cast<const uint64_t*>(&v)), "l"(*reinterpret_cast<const uint64_t*>(&acc)));
    return *reinterpret_cast<const float2*>(&r);
}

// The 8 factors of pairs 8g..8g+7 of one table row (shared or global memory).
__device__ __forceinline__ void rope_row8(const float2* row, int g, float2 (&wr)[4], float2 (&wi)[4]) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const float4 f = *reinterpret_cast<const float4*>(row + 8 * g + 2 * jj);
        wr[jj] = make_float2(f.x, f.z);
        wi[jj] = make_float2(f.y, f.w);
    }
}

struct OutSpec {
    void* out;
    int64_t o_bstride, o_hstride;
    uint32_t flags;
};

// One output element: BF16 acc/l (round to nearest even), or the FP32 partial row.
__device__ __forceinline__ void write_result(const OutSpec& o, int b, int qh, int dim, float acc, float m, float l) {
    if (o.flags & 1u) {
        float* r = static_cast<float*>(o.out) + (int64_t)b * o.o_bstride + (int64_t)qh * o.o_hstride;
        r[dim] = acc;
        if (dim == 0) {
            r[128] = m;
            r[129] = l;
            r[130] = 0.f;
            r[131] = 0.f;
        }
    } else {
        __nv_bfloat16* r = static_cast<__nv_bfloat16*>(o.out) + (int64_t)b * o.o_bstride + (int64_t)qh * o.o_hstride;
        r[dim] = __float2bfloat16_rn(acc / l);
    }
}

// Four consecutive output elements dim0 .. dim0+3 (dim0 a multiple of 4; rows are 16-byte aligned).
__device__ __forceinline__ void write_result4(const OutSpec& o, int b, int qh, int dim0, float4 acc, float m,
                                              float l) {
    if (o.flags & 1u) {
        float* r = static_cast<float*>(o.out) + (int64_t)b * o.o_bstride + (int64_t)qh * o.o_hstride;
        *reinterpret_cast<float4*>(r + dim0) = acc;
        if (dim0 == 0) *reinterpret_cast<float4*>(r + 128) = make_float4(m, l, 0.f, 0.f);
    } else {
        __nv_bfloat16* r = static_cast<__nv_bfloat16*>(o.out) + (int64_t)b * o.o_bstride + (int64_t)qh * o.o_hstride;
        const __nv_bfloat162 lo = __halves2bfloat162(__float2bfloat16_rn(acc.x / l), __float2bfloat16_rn(acc.y / l));
        const __nv_bfloat162 hi = __halves2bfloat162(__float2bfloat16_rn(acc.z / l), __float2bfloat16_rn(acc.w / l));
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t*>(&lo);
        w.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(r + dim0) = w;
    }
}

// RoPE constants the producer warp needs for pairs 2 lane and 2 lane + 1,
// read from the immutable table before the grid dependency wait.
struct ProducerRope {
    uint64_t step0, step1;  // Q0.64 turns per position
    float2 back_r, back_i;  // e^{-i theta kTileKeys}: one tile back
};

// Producer warp.  Lane 0 issues the group's 4 Q rows, then per tile one TMA
// box for K and one for V (88 rows of one head, whatever the K/V strides) into
// the shared-memory ring.  Unless K comes rotated, the whole warp also writes
// each stage's Q: RoPE is relative, so with T the tile's first key position
// and m the query position the score of key T + r is
//   Re sum_i Q_T,i conj(k_i e^{i theta_i r}),  Q_T = q e^{i theta (m - T)} * qscale,
// and the consumers rotate K by fixed per-lane factors e^{i theta r} only.  The
// warp computes Q_T once per tile (2 pairs of 4 heads per lane: the factor
// advances by one tile with a complex multiply, exactly every kReanchorTiles),
// stores it and arrives on the stage's full barrier a second time.  Returns
// once every copy into this CTA's shared memory has landed.
template <bool kKRotated>
__device__ __forceinline__ void produce_tiles(const DecodeArgs& a, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                             uint64_t* qbar, int b, int h, int hm, int64_t first_row, int n_tiles,
                                             int64_t q_minus_first, const ProducerRope& pr, int lane) {
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int t) {  // lane 0
        const int st = t % kStages;
        uint8_t* kd = smem + st * kStageBytes;
        uint8_t* vd = kd + kTileBytes;
        mbar_arrive_expect_tx(&full[st], 2 * kTileBytes);
        const int row = static_cast<int>(first_row + (int64_t)t * kTileKeys);
        const int c1 = a.kv_rows_inner ? row : hm, c2 = a.kv_rows_inner ? hm : row;
        tma_load_3d(kd, &a.kmap, 0, c1, c2, &full[st], pol);
        tma_load_3d(vd, &a.vmap, 0, c1, c2, &full[st], pol);
    };
    const int n_pre = min(n_tiles, kStages);
    if (lane == 0) {
        // The group's Q rows go first, ahead of the K/V stream; the first
        // stages' copies need no wait.
        mbar_arrive_expect_tx(qbar, kGroup * kRowBytes);
        for (int hq = 0; hq < kGroup; ++hq)
            bulk_load(smem + kOffQ + hq * kRowBytes,
                      a.q + (int64_t)b * a.q_bstride + (int64_t)(h * kGroup + hq) * a.q_hstride, kRowBytes, qbar,
                      pol);
        for (int t = 0; t < n_pre; ++t) issue(t);
    }
    int issued = n_pre, rotated = 0;  // tiles whose copies were issued / whose Q_T was written
    bool ok = true;
    if constexpr (!kKRotated) {
        ok = mbar_wait(qbar, 0);
        const uint8_t* qs = smem + kOffQ;
        float2 q_re[kGroup], q_im[kGroup];  // pairs 2 lane, 2 lane + 1 of each head (BF16, exact)
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq) {
            q_re[hq] = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(qs + hq * kRowBytes + 4 * lane));
            q_im[hq] = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(qs + hq * kRowBytes + 128 + 4 * lane));
        }
        float2 gr, gi;  // qscale e^{i theta (m - T)} of the two pairs
        auto exact = [&](int64_t pos) {
            const float2 f0 = rope_factor(pr.step0, pos), f1 = rope_factor(pr.step1, pos);
            gr = make_float2(f0.x * a.qscale, f1.x * a.qscale);
            gi = make_float2(f0.y * a.qscale, f1.y * a.qscale);
        };
        exact(q_minus_first);
        const int off = ((lane >> 1) & 1) * 32 + (lane >> 2) * 4 + 2 * (lane & 1);
        float* qt_base = reinterpret_cast<float*>(smem + kOffQt);
        for (int t = 0; t < n_tiles && ok; ++t) {
            const int st = t % kStages;
            if (t >= kStages) {
                bool w = true;
                if (lane == 0) {
                    w = mbar_wait(&empty[st], ((t / kStages) - 1) & 1);
                    if (w) issue(t);
                }
                if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                issued = t + 1;
            }
            float* qt = qt_base + st * kQtFloats;
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq) {
                float2 re, im;
                cmul2(q_re[hq], q_im[hq], gr, gi, re, im);
                *reinterpret_cast<float2*>(qt + hq * kHeadDim + off) = re;
                *reinterpret_cast<float2*>(qt + hq * kHeadDim + 64 + off) = im;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[st]);
            rotated = t + 1;
            if (((t + 1) % kReanchorTiles) == 0) {
                exact(q_minus_first - (int64_t)(t + 1) * kTileKeys);
            } else {
                float2 nr, ni;
                cmul2(gr, gi, pr.back_r, pr.back_i, nr, ni);
                gr = nr;
                gi = ni;
            }
        }
    } else if (lane == 0) {
        for (int t = kStages; t < n_tiles; ++t) {
            if (!mbar_wait(&empty[t % kStages], ((t / kStages) - 1) & 1)) {
                ok = false;
                break;
            }
            issue(t);
            issued = t + 1;
        }
    }
    if (lane != 0) return;
    if (!ok) atomicOr(a.ws_status, kDevStatusTimeout);
    // Do not leave while copies into this CTA's shared memory are in flight
    // (after a failed wait, complete the stages whose Q_T was not written).
    if (!kKRotated)
        for (int t = rotated; t < issued; ++t) mbar_arrive(&full[t % kStages]);
    mbar_wait(qbar, 0);
    for (int t = max(0, issued - kStages); t < issued; ++t) mbar_wait(&full[t % kStages], (t / kStages) & 1);
}

// ---------------------------------------------------------------------------
// decode_queue_kernel (a batch): its shared memory is decode_kernel's ring, P,
// alpha, RoPE and Q_T regions at the same offsets, and behind them
//   barriers  full/empty are decode_kernel's; here qbar[2] (two Q-row slots),
//             filled[2] and freed[2] (two item slots: the producer warp fills
//             one, the consumer warps free it once read)
//   Q rows    [2 slots][4 rows] BF16
//   items     [2 slots][kItemInts] ints
//   epilogue  the warps' partials and factors, outside the ring so that the
//             next item's tiles can land while it is in use.
// ---------------------------------------------------------------------------
constexpr int kItemInts = 16;
constexpr int kQueueOffBars = kSmemBytes;
constexpr int kQueueOffQ = kQueueOffBars + 6 * 8;
constexpr int kQueueOffItems = kQueueOffQ + 2 * kGroup * kRowBytes;
constexpr int kQueueOffEpi = kQueueOffItems + 2 * kItemInts * 4;
constexpr int kQueueEpiFloats = kConsumerWarps * kGroup * kPartialFloats + 2 * kConsumerWarps * kGroup + kGroup;
constexpr int kQueueSmemBytes = kQueueOffEpi + kQueueEpiFloats * 4;
static_assert(kQueueOffQ % 16 == 0 && kQueueOffEpi % 16 == 0, "16-byte aligned regions");
static_assert(kQueueSmemBytes <= 227 * 1024, "shared memory of one CTA");

// Producer warp of decode_queue_kernel, one item (a split of one KV head).
// Lane 0 issues the group's 4 Q rows into the slot `qrows` (barrier qbar),
// then per tile one TMA box for K and one for V into ring positions ring0,
// ring0 + 1, ... (stage p % kStages), first waiting for the stage's release
// once the ring has gone round.  Unless K comes rotated the warp also writes
// each stage's Q_T and arrives on its full barrier a second time, as
// produce_tiles does.  `issued` and `rotated` end as one past the last ring
// position whose copies were issued and whose Q_T was written; false after a
// timed-out wait.
template <bool kKRotated>
__device__ __forceinline__ bool produce_item(const DecodeArgs& a, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                             uint64_t* qbar, uint32_t qparity, uint8_t* qrows, int b, int h, int hm,
                                             int64_t first_row, int n_tiles, int64_t q_minus_first,
                                             const ProducerRope& pr, int lane, int ring0, int& issued, int& rotated) {
    const uint64_t pol = l2_evict_first_policy();
    if (lane == 0) {
        // The group's Q rows go first, ahead of the item's K/V stream.
        mbar_arrive_expect_tx(qbar, kGroup * kRowBytes);
        for (int hq = 0; hq < kGroup; ++hq)
            bulk_load(qrows + hq * kRowBytes,
                      a.q + (int64_t)b * a.q_bstride + (int64_t)(h * kGroup + hq) * a.q_hstride, kRowBytes, qbar,
                      pol);
    }
    float2 q_re[kGroup], q_im[kGroup];  // pairs 2 lane, 2 lane + 1 of each head (BF16, exact)
    float2 gr, gi;                      // qscale e^{i theta (m - T)} of the two pairs
    auto exact = [&](int64_t pos) {
        const float2 f0 = rope_factor(pr.step0, pos), f1 = rope_factor(pr.step1, pos);
        gr = make_float2(f0.x * a.qscale, f1.x * a.qscale);
        gi = make_float2(f0.y * a.qscale, f1.y * a.qscale);
    };
    if (!kKRotated) exact(q_minus_first);
    const int off = ((lane >> 1) & 1) * 32 + (lane >> 2) * 4 + 2 * (lane & 1);
    float* qt_base = reinterpret_cast<float*>(smem + kOffQt);
    for (int t = 0; t < n_tiles; ++t) {
        const int p = ring0 + t, st = p % kStages;
        bool w = true;
        if (lane == 0) {
            if (p >= kStages) w = mbar_wait(&empty[st], ((p / kStages) - 1) & 1);
            if (w) {
                uint8_t* kd = smem + st * kStageBytes;
                uint8_t* vd = kd + kTileBytes;
                mbar_arrive_expect_tx(&full[st], 2 * kTileBytes);
                const int row = static_cast<int>(first_row + (int64_t)t * kTileKeys);
                const int c1 = a.kv_rows_inner ? row : hm, c2 = a.kv_rows_inner ? hm : row;
                tma_load_3d(kd, &a.kmap, 0, c1, c2, &full[st], pol);
                tma_load_3d(vd, &a.vmap, 0, c1, c2, &full[st], pol);
            }
        }
        if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) return false;
        issued = p + 1;
        if constexpr (!kKRotated) {
            if (t == 0) {  // the tile's copies are on their way: now wait for the Q rows
                const bool okq = mbar_wait(qbar, qparity);
                if (!__all_sync(0xffffffffu, okq)) return false;
#pragma unroll
                for (int hq = 0; hq < kGroup; ++hq) {
                    q_re[hq] = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(qrows + hq * kRowBytes + 4 * lane));
                    q_im[hq] =
                        bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(qrows + hq * kRowBytes + 128 + 4 * lane));
                }
            }
            float* qt = qt_base + st * kQtFloats;
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq) {
                float2 re, im;
                cmul2(q_re[hq], q_im[hq], gr, gi, re, im);
                *reinterpret_cast<float2*>(qt + hq * kHeadDim + off) = re;
                *reinterpret_cast<float2*>(qt + hq * kHeadDim + 64 + off) = im;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[st]);
            rotated = p + 1;
            if (((t + 1) % kReanchorTiles) == 0) {
                exact(q_minus_first - (int64_t)(t + 1) * kTileKeys);
            } else {
                float2 nr, ni;
                cmul2(gr, gi, pr.back_r, pr.back_i, nr, ni);
                gr = nr;
                gi = ni;
            }
        }
    }
    // An item without keys: its Q-row copy must still complete before the
    // slot is used again.
    if (!kKRotated && n_tiles == 0 && !__all_sync(0xffffffffu, mbar_wait(qbar, qparity))) return false;
    return true;
}

// Cluster epilogue of a single sequence: the n splits (CTA ranks 0..n-1) of KV
// head h each hold their partial (acc[128], m, l per Q head) at `cpart`.  The
// 512 outputs form 16 groups of 32 (one Q head, 32 dims); group w*n + rank goes
// to warp w of CTA `rank`, one output per lane, merged as
//   M = max m_s,  L = sum 2^(m_s - M) l_s,  O = sum 2^(m_s - M) acc_s
// with split s's (m, l) loaded by lane s.
constexpr int kMaxClusterSplits = 16;
static_assert(kConsumerWarps * 2 >= kOutputs / 32, "two splits cover the 16 output groups");

__device__ __forceinline__ void cluster_merge(int n, int rank, int c, int lane, const float* cpart,
                                              const OutSpec& direct, int h) {
    cluster_sync_all();  // every split's partial is in its shared memory
    const int grp = c * n + rank;
    if (grp < kOutputs / 32) {
        const int hq = grp >> 2, dim = (grp & 3) * 32 + lane;
        const float* row = cpart + hq * kPartialFloats;
        float ms = -INFINITY, ls = 0.f;
        if (lane < n) {
            const float2 x = ld_cluster_f32x2(cluster_map(row + 128, lane));
            ms = x.x;
            ls = x.y;
        }
        float vals[kMaxClusterSplits];
#pragma unroll
        for (int s = 0; s < kMaxClusterSplits; ++s) vals[s] = s < n ? ld_cluster_f32(cluster_map(row + dim, s)) : 0.f;
        float M = ms;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float Mu = M == -INFINITY ? 0.f : M;
        const float f = lane < n ? exp2f(ms - Mu) : 0.f;
        float L = ls * f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < kMaxClusterSplits; ++s) o4[s & 3] = fmaf(vals[s], __shfl_sync(0xffffffffu, f, s), o4[s & 3]);
        write_result(direct, 0, h * kGroup + hq, dim, (o4[0] + o4[1]) + (o4[2] + o4[3]), M, L);
    }
    cluster_sync_all();  // no CTA leaves while another may still read its partial
}

// Merge of a single sequence's n <= 32 splits by the last split CTA of KV head
// h to finish (the others return): each CTA's partial is in the workspace; an
// arrival counter per KV head (release fence, then atomic add; zeroed again by
// the last arrival) picks the last one, which reads every split's (m, l) and
// acc column from L2 in one round trip, then
//   M = max m_s,  L = sum 2^(m_s - M) l_s,  O = sum 2^(m_s - M) acc_s
// with warp hq reducing head hq's (m, l) over lanes s.  Consumer thread tid
// owns outputs tid and tid + kConsumerThreads of the 512.
constexpr int kLastMergeMaxSplits = 32;
constexpr int kMergeBatch = 20;  // splits whose acc values a thread loads before the first use
static_assert(2 * kConsumerThreads >= kOutputs, "two outputs per consumer thread cover the head group");
static_assert(kConsumerWarps >= kGroup, "one warp per Q head reduces (m, l)");

// Arrival of one split: releases the CTA's partial stores (ordered before it
// through the CTA barrier; release is cumulative) and, for the last split,
// acquires every earlier split's -- one acq_rel atomic instead of a fence on
// either side of a relaxed one.
__device__ __forceinline__ uint32_t arrive_acq_rel_gpu(uint32_t* p) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
    return old;
}

constexpr int kLastMergeScratchFloats = kGroup * kLastMergeMaxSplits + 2 * kGroup;

// Long-context split across GPUs, fused into the decode: the CTA that holds
// this rank's merged rows of Q heads 4h..4h+3 (acc[128], m, l in shared
// memory) pushes them into every rank's exchange buffer
// (push_rows[e & 1][rank]) as 64-bit words that each carry the value and the
// epoch e: one NVLink write per word carries its own flag, so the data needs
// no fence and no separate flag store.  Each thread then polls, in its OWN
// buffer (bounded), the words of the outputs it merges, for every source
// rank, and merges
//   M = max m_r, O = sum 2^(m_r - M) acc_r, L = sum 2^(m_r - M) l_r,
// writing BF16 O / L; the last of the eight heads advances the epoch.  Rows of
// epoch e are rewritten at e + 2 only: by then every peer has published e + 1,
// which it does after finishing epoch e; a stale word carries e - 2 and is
// never mistaken for e.
__device__ __forceinline__ void st_word_sys(uint64_t* p, float v, uint32_t e) {
    const uint64_t w = ((uint64_t)e << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word_sys(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Word p as first loaded (`w`), or once it carries epoch e: a bounded wait only
// for a word that had not arrived yet; ok turns false on expiry and stays false.
__device__ __forceinline__ float word_value(uint64_t w, const uint64_t* p, uint32_t e, bool& ok) {
    if ((uint32_t)(w >> 32) != e && ok) {
        const long long t0 = clock64();
        do {
            w = ld_word_sys(p);
            if (clock64() - t0 > kWaitTimeoutCycles) {
                ok = false;
                break;
            }
        } while ((uint32_t)(w >> 32) != e);
    }
    return __uint_as_float((uint32_t)w);
}

__device__ __forceinline__ void exchange_and_finish(const DecodeArgs& a, int h, int tid, const float* rows,
                                                    int* info, const OutSpec& direct) {
    uint8_t* mine = reinterpret_cast<uint8_t*>(a.peer_bases[a.rank]);
    uint32_t* hdr = reinterpret_cast<uint32_t*>(mine);
    const size_t push = peer_push_offset(1);
    if (tid == 0) info[3] = (int)(*reinterpret_cast<volatile uint32_t*>(hdr) + 1u);
    named_barrier_sync(1, kConsumerThreads);
    const uint32_t e = (uint32_t)info[3];
    // Words of (source rank r, Q head 4h + hq) of parity e & 1 in any rank's push area.
    auto push_row = [&](uint8_t* base, int r) {
        return reinterpret_cast<uint64_t*>(base + push + kPushFlagsBytes) +
               (((size_t)(e & 1u) * kMaxPeers + r) * kNumQHeads + (size_t)h * kGroup) * kPushRowWords;
    };
    for (int p = 0; p < a.world; ++p) {
        uint64_t* dst = push_row(reinterpret_cast<uint8_t*>(a.peer_bases[p]), a.rank);
        for (int i = tid; i < kGroup * kPushRowWords; i += kConsumerThreads)
            st_word_sys(dst + i, rows[(i / kPushRowWords) * kPartialFloats + i % kPushRowWords], e);
    }
    bool ok = true;
    for (int o = tid; o < kOutputs; o += kConsumerThreads) {
        const int hq = o >> 7, dim = o & 127;
        // All 3 x world words are loaded before any is examined, so their
        // latencies overlap; only a word that has not arrived is polled again.
        uint64_t wm[kMaxPeers], wl[kMaxPeers], wa[kMaxPeers];
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r < a.world) {
                const uint64_t* row = push_row(mine, r) + hq * kPushRowWords;
                wm[r] = ld_word_sys(row + kHeadDim);
                wl[r] = ld_word_sys(row + kHeadDim + 1);
                wa[r] = ld_word_sys(row + dim);
            }
        }
        float mr[kMaxPeers], lr[kMaxPeers], ar[kMaxPeers];
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r < a.world) {
                const uint64_t* row = push_row(mine, r) + hq * kPushRowWords;
                mr[r] = word_value(wm[r], row + kHeadDim, e, ok);
                lr[r] = word_value(wl[r], row + kHeadDim + 1, e, ok);
                ar[r] = word_value(wa[r], row + dim, e, ok);
            }
        }
        if (!ok) break;
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)
            if (r < a.world) M = fmaxf(M, mr[r]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r < a.world) {
                const float f = exp2f(mr[r] - Mu);
                L = fmaf(lr[r], f, L);
                O = fmaf(ar[r], f, O);
            }
        }
        write_result(direct, 0, h * kGroup + hq, dim, O, M, L);
    }
    if (!ok) atomicOr(a.ws_status, kDevStatusTimeout);
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(hdr + 1, 1u) == (uint32_t)(kNumKVHeads - 1)) {
            hdr[1] = 0u;
            *reinterpret_cast<volatile uint32_t*>(hdr) = e;
        }
    }
}

__device__ __forceinline__ void last_split_merge(const DecodeArgs& a, int n, int h, int tid, float* sh, int* flag,
                                                 const OutSpec& direct, float* xrows, int* info) {
    named_barrier_sync(1, kConsumerThreads);  // every partial store of this CTA is issued
    if (tid == 0) {
        const uint32_t prev = arrive_acq_rel_gpu(a.ws_arrivals + h);
        const int last = prev == (uint32_t)(n - 1);
        if (last) a.ws_arrivals[h] = 0u;  // the next call's kernel starts after this one completes
        *flag = last;
    }
    named_barrier_sync(1, kConsumerThreads);
    if (*flag == 0) return;

    const int warp = tid >> 5, lane = tid & 31;
    const int64_t sstride = (int64_t)kNumKVHeads * kGroup * kPartialFloats;
    const float* base = a.ws_partials + (int64_t)h * kGroup * kPartialFloats;
    float* fsh = sh;                                  // [hq][s]  2^(m_s - M)
    float* tot = fsh + kGroup * kLastMergeMaxSplits;  // [hq]     (M, L)
    float2 ml = make_float2(-INFINITY, 0.f);
    if (warp < kGroup && lane < n) ml = __ldcg(reinterpret_cast<const float2*>(base + lane * sstride + warp * kPartialFloats + 128));
    const int o1 = tid + kConsumerThreads;
    const bool has1 = o1 < kOutputs;
    const float* p0 = base + (tid >> 7) * kPartialFloats + (tid & 127);
    const float* p1 = base + ((has1 ? o1 : 0) >> 7) * kPartialFloats + (o1 & 127);
    float v0[kMergeBatch], v1[kMergeBatch];
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
        v0[j] = j < n ? __ldcg(p0 + j * sstride) : 0.f;
        v1[j] = has1 && j < n ? __ldcg(p1 + j * sstride) : 0.f;
    }
    if (warp < kGroup) {
        float M = ml.x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float f = lane < n ? exp2f(ml.x - (M == -INFINITY ? 0.f : M)) : 0.f;
        float L = ml.y * f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        fsh[warp * kLastMergeMaxSplits + lane] = f;
        if (lane == 0) {
            tot[2 * warp] = M;
            tot[2 * warp + 1] = L;
        }
    }
    named_barrier_sync(1, kConsumerThreads);
    auto finish = [&](int o, const float (&v)[kMergeBatch], const float* p) {
        const int hq = o >> 7;
        const float* f = fsh + hq * kLastMergeMaxSplits;
        float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < kMergeBatch; ++j) o4[j & 3] = fmaf(v[j], f[j], o4[j & 3]);  // f[j] = 0 past n
        float rest = 0.f;
        for (int s = kMergeBatch; s < n; ++s) rest = fmaf(__ldcg(p + s * sstride), f[s], rest);
        const float O = ((o4[0] + o4[1]) + (o4[2] + o4[3])) + rest;
        if (a.world > 1) {  // this rank's merged rows go to the cross-GPU exchange
            xrows[hq * kPartialFloats + (o & 127)] = O;
            if ((o & 127) == 0) {
                xrows[hq * kPartialFloats + kHeadDim] = tot[2 * hq];
                xrows[hq * kPartialFloats + kHeadDim + 1] = tot[2 * hq + 1];
            }
        } else {
            write_result(direct, 0, h * kGroup + hq, o & 127, O, tot[2 * hq], tot[2 * hq + 1]);
        }
    };
    finish(tid, v0, p0);
    if (has1) finish(o1, v1, p1);
    if (a.world > 1) {
        named_barrier_sync(1, kConsumerThreads);
        exchange_and_finish(a, h, tid, xrows, info, direct);
    }
}

// Epilogue shared memory (in the drained ring): warp partials, the split's merged
// partial, the last-split merge's scratch, the warp factors.
static_assert((kConsumerWarps * kGroup * kPartialFloats + kGroup * kPartialFloats + kLastMergeScratchFloats +
               2 * kConsumerWarps * kGroup + kGroup + kGroup * kPartialFloats) * 4 <= kOffBars,
              "epilogue buffers fit the ring");

// kKRotated: the K rows are stored already rotated (GQA_FLAG_K_ROTATED, RoPE
// applied when they were appended); only Q is rotated here.
template <bool kKRotated>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* empty = full + kStages;
    float* pbuf = reinterpret_cast<float*>(smem + kOffP);
    float* abuf = reinterpret_cast<float*>(smem + kOffAlpha);
    float2* rope = reinterpret_cast<float2*>(smem + kOffRope);
    int* info = reinterpret_cast<int*>(smem + kOffInfo);
    const RopeTable* rt = a.rope;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tid = threadIdx.x;
    const bool clustered = a.cluster > 0;  // grid (splits, heads), one cluster per head
    // KV head: h in the call's numbering (Q rows, output rows, partials,
    // arrival counters), hm = h - head0 in the K/V tensor maps.
    const int hm = clustered ? (int)blockIdx.y : (int)(blockIdx.x % a.n_heads);
    const int h = a.head0 + hm;
    const int gsplit = clustered ? (int)blockIdx.x : (int)(blockIdx.x / a.n_heads);
    const bool single = a.descs == nullptr;

    uint64_t* qbar = empty + kStages;
    const uint8_t* qs = smem + kOffQ;
    const int c = warp;
    const int slot = lane >> 3;  // key within the group of 4 a step handles
    const int g = lane & 7;      // pairs 8g .. 8g+7 (dims 8g..8g+7 and 64+8g..64+8g+7)
    const int hh = g >> 1;       // Q head whose score this lane holds after the reduction

    // ---- set-up that reads only the argument block: before the dependency wait
    if (tid == kConsumerThreads) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kKRotated ? 1 : 2);  // + the producer warp's Q_T
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(qbar, 1);
        fence_barrier_init();
        prefetch_tensormap(&a.kmap);
        prefetch_tensormap(&a.vmap);
    }
    // RoPE constants from the immutable table (L2-resident after the first
    // CTA).  Unrotated K: each consumer lane's fixed factors e^{i theta r} of
    // its key r of a tile in steps 0 and 1, and the producer warp's constants
    // for Q_T.  Pre-rotated K: the consumers rotate Q once, at QUERY_POSITION
    // (computed exactly, one factor per thread of the first 64).
    float2 qfr[4], qfi[4], kfr[kSteps][4], kfi[kSteps][4];
    ProducerRope prope{};
    if (!kKRotated && warp < kConsumerWarps) {
#pragma unroll
        for (int step = 0; step < kSteps; ++step)
            rope_row8(rt->key_off[c * kKeysPerWarp + step * 4 + slot], g, kfr[step], kfi[step]);
    }
    if (!kKRotated && warp == kConsumerWarps) {
        prope.step0 = rt->step[2 * lane];
        prope.step1 = rt->step[2 * lane + 1];
        const float2 t0 = rt->rot_tile[2 * lane], t1 = rt->rot_tile[2 * lane + 1];
        prope.back_r = make_float2(t0.x, t1.x);
        prope.back_i = make_float2(-t0.y, -t1.y);
    }
    auto lane_rope = [&](int qpos) {
        if (tid < kPairs) rope[kRopeQ * kPairs + tid] = rope_factor(rt->step[tid], qpos);
        named_barrier_sync(1, kConsumerThreads);
        rope_row8(rope + kRopeQ * kPairs, g, qfr, qfi);
        if (a.flags & GQA_FLAG_Q_ROTATED) {  // Q supplied rotated: identity factors (exact)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                qfr[jj] = make_float2(1.f, 1.f);
                qfi[jj] = make_float2(0.f, 0.f);
            }
        }
    };
    if (kKRotated && single && warp < kConsumerWarps) lane_rope(a.single.query_position);
    // A single sequence's split needs no memory read to know its keys: pull its
    // Q rows and first K/V tiles into L2 while the previous kernel in the stream
    // finishes (its loads below then hit L2).
    if (single && tid == kConsumerThreads) {
        const int n_keys = seq_key_count(a.single);
        const int key0 = gsplit * a.chunk;
        const int cnt = max(0, min(a.chunk, n_keys - key0));
        const int n_pre = min((cnt + kTileKeys - 1) / kTileKeys, kStages);
        for (int hq = 0; hq < kGroup; ++hq) bulk_prefetch_l2(a.q + (int64_t)(h * kGroup + hq) * a.q_hstride, kRowBytes);
        for (int t = 0; t < n_pre; ++t) {
            const int row = static_cast<int>(a.single.kv_start + key0 + (int64_t)t * kTileKeys);
            tma_prefetch_3d(&a.kmap, 0, a.kv_rows_inner ? row : hm, a.kv_rows_inner ? hm : row);
            tma_prefetch_3d(&a.vmap, 0, a.kv_rows_inner ? row : hm, a.kv_rows_inner ? hm : row);
        }
    }
    allow_dependent_launch();
    grid_dependency_wait();

    // ---- which (sequence, split) this CTA owns, computed by the producer warp,
    // which goes on to issue the loads at once; the consumers pick the result up
    // through named barrier 2.  A batch runs every sequence's full-chunk splits
    // first and the shorter last splits after them, so that those fill the last
    // wave; partials are stored by the logical index prefix_splits[b] + split,
    // contiguous per sequence for the split merge.
    if (warp == kConsumerWarps) {
        int b = 0, split = gsplit, logical = gsplit;
        if (!single) {
            // Sequence b has full_b = keys / chunk full splits and
            // seq_splits - full_b (0 or 1) shorter last ones.
            auto counts = [&](int bb, int& nf, int& np) {
                nf = np = 0;
                if (bb < a.batch) {
                    const SeqDesc db = a.descs[bb];
                    nf = seq_key_count(db) / a.chunk;
                    np = seq_splits(db, a.chunk) - nf;
                }
            };
            auto scan = [&](int v) {
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, v, o);
                    if (lane >= o) v += t;
                }
                return v;
            };
            int total_full = 0;
            for (int b0 = 0; b0 < a.batch; b0 += 32) {
                int nf, np;
                counts(b0 + lane, nf, np);
                total_full += __shfl_sync(0xffffffffu, scan(nf), 31);
            }
            const bool in_full = gsplit < total_full;
            const int target = in_full ? gsplit : gsplit - total_full;
            int base = 0, sbase = 0;  // splits of the chosen kind / of any kind before b0
            b = -1;
            for (int b0 = 0; b0 < a.batch && b < 0; b0 += 32) {
                int nf, np;
                counts(b0 + lane, nf, np);
                const int nk = in_full ? nf : np;
                const int incl = scan(nk), sincl = scan(nf + np);
                const int excl = incl - nk;
                const bool hit = b0 + lane < a.batch && target >= base + excl && target < base + incl;
                const unsigned m = __ballot_sync(0xffffffffu, hit);
                if (m) {
                    const int src = __ffs(m) - 1;
                    b = b0 + src;
                    const int nf_src = __shfl_sync(0xffffffffu, nf, src);
                    split = in_full ? target - base - __shfl_sync(0xffffffffu, excl, src) : nf_src;
                    const int sexcl = __shfl_sync(0xffffffffu, sincl - (nf + np), src);
                    logical = sbase + sexcl + split;
                }
                base += __shfl_sync(0xffffffffu, incl, 31);
                sbase += __shfl_sync(0xffffffffu, sincl, 31);
            }
        }
        if (lane == 0) {
            info[0] = b;
            info[1] = split;
            info[5] = logical;
        }
        __syncwarp();
        named_barrier_arrive(2, kThreads);
    } else {
        named_barrier_sync(2, kThreads);
    }
    const int b = info[0];
    const int split = info[1];
    const int lsplit = info[5];  // storage index of this split's partial
    if (b < 0) return;  // grid larger than the plan: nothing to do (uniform per CTA)
    const SeqDesc d = single ? a.single : a.descs[b];
    const int n_keys = seq_key_count(d);
    const int n_split = seq_splits(d, a.chunk);
    const int key0 = split * a.chunk;
    const int cnt = max(0, min(a.chunk, n_keys - key0));
    const int n_tiles = (cnt + kTileKeys - 1) / kTileKeys;
    const int64_t first_pos = (int64_t)d.pos_begin + key0;
    const int64_t first_row = d.kv_start + key0;

    // The split merge finds each sequence's splits here.
    if (!clustered && split == 0 && hm == 0 && tid == 0 && n_split > 1) a.ws_seqinfo[b] = make_int2(lsplit, n_split);

    // ======================= producer warp =======================
    // In a cluster the whole warp also takes part in the epilogue's two cluster
    // barriers.
    if (warp == kConsumerWarps) {
        // m - T of the first tile (Q supplied rotated: m = 0).
        const int64_t q_minus_first =
            ((a.flags & GQA_FLAG_Q_ROTATED) ? 0 : (int64_t)d.query_position) - first_pos;
        produce_tiles<kKRotated>(a, smem, full, empty, qbar, b, h, hm, first_row, n_tiles, q_minus_first, prope,
                                 lane);
        if (clustered) {
            __syncwarp();
            cluster_sync_all();  // partials published
            cluster_sync_all();  // partials read: shared memory may be released
        }
        return;
    }

    // ======================= consumer warps =======================
    const int qpos = d.query_position;
    if (a.mask_out != nullptr && split == 0 && hm == 0) {
        const int n_pad = ((d.seq_len + a.kv_block_len - 1) / a.kv_block_len) * a.kv_block_len;
        for (int p = tid; p < n_pad; p += kConsumerThreads)
            a.mask_out[(int64_t)b * a.mask_stride + p] = key_valid(p, d.seq_len, qpos) ? 1 : 0;
    }
    if (kKRotated && !single) lane_rope(qpos);

    // Q pre-scaled by scale*log2(e): rotated at QUERY_POSITION once (K
    // pre-rotated), or to each tile's first key by the producer (loaded per
    // tile in qk_tile).  Register slot j of a lane holds Q head j ^ hh, so
    // that the score reduction below needs no per-lane selects (each lane
    // keeps slots 0/1 and sends 2/3).
    float2 qr[kGroup][4], qi[kGroup][4];
    bool ok = kKRotated ? mbar_wait(qbar, 0) : true;
#pragma unroll
    for (int j = 0; j < kGroup && kKRotated; ++j) {
        const uint8_t* qrow = qs + (j ^ hh) * kRowBytes;
        const uint4 xr = *reinterpret_cast<const uint4*>(qrow + g * 16);
        const uint4 xi = *reinterpret_cast<const uint4*>(qrow + 128 + g * 16);
        const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
        const uint32_t yw[4] = {xi.x, xi.y, xi.z, xi.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            float2 re, im;
            cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), qfr[jj], qfi[jj], re, im);
            qr[j][jj] = __fmul2_rn(re, f2(a.qscale));
            qi[j][jj] = __fmul2_rn(im, f2(a.qscale));
        }
    }

    float m_run = -INFINITY;  // running max (log2 units) of head hh
    float l_run = 0.f;        // running sum of this lane's key slot for head hh
    float2 acc0[kGroup], acc1[kGroup];  // dims (4*lane, +1) and (4*lane+2, +3) of each head
#pragma unroll
    for (int hq = 0; hq < kGroup; ++hq) acc0[hq] = acc1[hq] = make_float2(0.f, 0.f);
    // Per-warp double buffer of probabilities [2][keys][4 heads] and rescales [2][4].
    float* pw = pbuf + c * 2 * (kKeysPerWarp * kGroup);
    float* aw = abuf + c * 2 * kGroup;

    // Scores of this warp's keys of tile t: RoPE of K, Q.K for the 4 heads,
    // reduction over the 8 lanes of each key.  Keys [key0, key0 + cnt) all
    // satisfy key_valid() (they lie in [0, min(SEQ_LEN, QUERY_POSITION + 1)));
    // rows past them are masked.
    auto qk_tile = [&](int t, float (&sc)[kSteps]) {
        const uint8_t* kt = smem + (t % kStages) * kStageBytes;
        const int rows = min(kTileKeys, cnt - t * kTileKeys);
        if constexpr (!kKRotated) {
            const float* qt = reinterpret_cast<const float*>(smem + kOffQt) + (t % kStages) * kQtFloats;
#pragma unroll
            for (int j = 0; j < kGroup; ++j) {
                const float* row = qt + (j ^ hh) * kHeadDim + 4 * g;
                const float4 r0 = *reinterpret_cast<const float4*>(row);
                const float4 r1 = *reinterpret_cast<const float4*>(row + 32);
                const float4 i0 = *reinterpret_cast<const float4*>(row + 64);
                const float4 i1 = *reinterpret_cast<const float4*>(row + 96);
                qr[j][0] = make_float2(r0.x, r0.y);
                qr[j][1] = make_float2(r0.z, r0.w);
                qr[j][2] = make_float2(r1.x, r1.y);
                qr[j][3] = make_float2(r1.z, r1.w);
                qi[j][0] = make_float2(i0.x, i0.y);
                qi[j][1] = make_float2(i0.z, i0.w);
                qi[j][2] = make_float2(i1.x, i1.y);
                qi[j][3] = make_float2(i1.z, i1.w);
            }
        }
#pragma unroll
        for (int step = 0; step < kSteps; ++step) {
            const int r = c * kKeysPerWarp + step * 4 + slot;
            const uint4 kre = *reinterpret_cast<const uint4*>(kt + r * kRowBytes + g * 16);
            const uint4 kim = *reinterpret_cast<const uint4*>(kt + r * kRowBytes + 128 + g * 16);
            const uint32_t xw[4] = {kre.x, kre.y, kre.z, kre.w};
            const uint32_t yw[4] = {kim.x, kim.y, kim.z, kim.w};
            float2 rr[4], ri[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                if constexpr (kKRotated) {
                    rr[jj] = bf16x2_to_float2(xw[jj]);
                    ri[jj] = bf16x2_to_float2(yw[jj]);
                } else {
                    cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), kfr[step][jj], kfi[step][jj], rr[jj],
                          ri[jj]);
                }
            }
            float s[kGroup];
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq) {
                float2 acc = __fmul2_rn(qr[hq][0], rr[0]);
                acc = __ffma2_rn(qi[hq][0], ri[0], acc);
#pragma unroll
                for (int jj = 1; jj < 4; ++jj) {
                    acc = __ffma2_rn(qr[hq][jj], rr[jj], acc);
                    acc = __ffma2_rn(qi[hq][jj], ri[jj], acc);
                }
                s[hq] = acc.x + acc.y;
            }
            // Lanes l and l^4 hold the same heads in swapped slot pairs, lanes l
            // and l^2 in swapped slots: keep 0/1, send 2/3; keep 0, send 1.
            const float t0 = s[0] + __shfl_xor_sync(0xffffffffu, s[2], 4);
            const float t1 = s[1] + __shfl_xor_sync(0xffffffffu, s[3], 4);
            float u = t0 + __shfl_xor_sync(0xffffffffu, t1, 2);
            u += __shfl_xor_sync(0xffffffffu, u, 1);
            sc[step] = r < rows ? u : -INFINITY;
        }
    };

    // Online softmax of head hh over this warp's keys of one tile, in
    // registers: the probabilities pv and the rescale alpha of the running sums.
    auto softmax_tile = [&](const float (&sc)[kSteps], float (&pv)[kSteps], float& alpha) {
        float mx = sc[0];
#pragma unroll
        for (int step = 1; step < kSteps; ++step) mx = fmaxf(mx, sc[step]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run, mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        alpha = fast_exp2(m_run - m_use);
        float psum = 0.f;
#pragma unroll
        for (int step = 0; step < kSteps; ++step) {
            pv[step] = fast_exp2(sc[step] - m_use);
            psum += pv[step];
        }
        l_run = l_run * alpha + psum;
        m_run = m_new;
    };
    // Stores p and the rescale into the warp's buffer `buf`; the caller's
    // __syncwarp publishes them to the warp.
    auto publish = [&](const float (&pv)[kSteps], float alpha, int buf) {
        float* pb = pw + buf * (kKeysPerWarp * kGroup);
        if ((g & 1) == 0) {
#pragma unroll
            for (int step = 0; step < kSteps; ++step) pb[(step * 4 + slot) * kGroup + hh] = pv[step];
            if (slot == 0) aw[buf * kGroup + hh] = alpha;
        }
    };

    // acc = acc * alpha + sum_k p_k * V_k over this warp's keys of tile t.
    // In the split's last tile, rows past its keys may hold anything (even
    // NaN): their probabilities are 0, and each lane zeroes the 8 bytes of
    // those rows that it reads itself, so no other lane is involved.
    auto pv_tile = [&](int t, int buf, bool last) {
        uint8_t* vt = smem + (t % kStages) * kStageBytes + kTileBytes;
        if (last) {
            const int nr = min(kTileKeys, cnt - t * kTileKeys) - c * kKeysPerWarp;
#pragma unroll
            for (int rr = 0; rr < kKeysPerWarp; ++rr)
                if (rr >= nr)
                    *reinterpret_cast<uint2*>(vt + (c * kKeysPerWarp + rr) * kRowBytes + lane * 8) = make_uint2(0u, 0u);
        }
        const float* pb = pw + buf * (kKeysPerWarp * kGroup);
        const float4 al = *reinterpret_cast<const float4*>(aw + buf * kGroup);
        const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq) {
            acc0[hq] = __fmul2_rn(acc0[hq], f2(alv[hq]));
            acc1[hq] = __fmul2_rn(acc1[hq], f2(alv[hq]));
        }
#pragma unroll
        for (int rr = 0; rr < kKeysPerWarp; ++rr) {
            const float4 p4 = *reinterpret_cast<const float4*>(pb + rr * kGroup);
            const uint2 vv = *reinterpret_cast<const uint2*>(vt + (c * kKeysPerWarp + rr) * kRowBytes + lane * 8);
            const float2 v0 = bf16x2_to_float2(vv.x), v1 = bf16x2_to_float2(vv.y);
            const float pk[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq) {
                acc0[hq] = ffma2_bcast(pk[hq], v0, acc0[hq]);
                acc1[hq] = ffma2_bcast(pk[hq], v1, acc1[hq]);
            }
        }
    };

    // Software pipeline: one iteration computes the scores and the softmax of
    // tile t and the P.V of tile t-1, with no branch or warp barrier between
    // them, so that the two independent instruction streams interleave; the
    // probabilities of tile t are stored after the P.V loads of tile t-1 (a
    // different buffer) and published by one __syncwarp.
    if (ok && n_tiles > 0) {
        if (mbar_wait(&full[0], 0)) {
            float sc[kSteps], pv[kSteps], alpha;
            qk_tile(0, sc);
            softmax_tile(sc, pv, alpha);
            publish(pv, alpha, 0);
            __syncwarp();
        } else {
            ok = false;
        }
    }
    for (int t = 1; t < n_tiles && ok; ++t) {
        if (!mbar_wait(&full[t % kStages], (t / kStages) & 1)) {
            ok = false;
            break;
        }
        float sc[kSteps], pv[kSteps], alpha;
        qk_tile(t, sc);
        softmax_tile(sc, pv, alpha);
        pv_tile(t - 1, (t - 1) & 1, false);
        publish(pv, alpha, t & 1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[(t - 1) % kStages]);
    }
    if (ok && n_tiles > 0) {
        pv_tile(n_tiles - 1, (n_tiles - 1) & 1, true);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[(n_tiles - 1) % kStages]);
    }
    if (!ok && lane == 0) atomicOr(a.ws_status, kDevStatusTimeout);

    l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);

    // ---- merge the warps through shared memory (the ring is free now)
    named_barrier_sync(1, kConsumerThreads);
    float* cb = reinterpret_cast<float*>(smem);
    {
        float* mine = cb + c * kGroup * kPartialFloats;
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq)
            *reinterpret_cast<float4*>(mine + hq * kPartialFloats + 4 * lane) =
                make_float4(acc0[hq].x, acc0[hq].y, acc1[hq].x, acc1[hq].y);
        if (slot == 0 && (g & 1) == 0) {
            mine[hh * kPartialFloats + 128] = m_run;
            mine[hh * kPartialFloats + 129] = l_run;
        }
    }
    named_barrier_sync(1, kConsumerThreads);

    const OutSpec direct{a.out, a.o_bstride, a.o_hstride, a.flags};
    // Shared memory behind the warp partials: the split's merged partial (for a
    // cluster), the last-split merge's scratch, and the warp factors.
    float* cpart = cb + kConsumerWarps * kGroup * kPartialFloats;
    float* lsm = cpart + kGroup * kPartialFloats;
    float* wf = lsm + kLastMergeScratchFloats;  // [w][hq]  2^(m_w - M)
    float* wl = wf + kConsumerWarps * kGroup;   // [w][hq]  l_w * 2^(m_w - M)
    float* wm = wl + kConsumerWarps * kGroup;   // [hq]     M
    float* xrows = wm + kGroup;                 // [hq][132] this rank's rows for the cross-GPU exchange
    const bool exchange = a.world > 1;
    // Factors once per (warp, head): thread t < 44 owns warp t / 4, head t % 4.
    if (tid < kConsumerWarps * kGroup) {
        const int hq = tid & 3;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cb[(w * kGroup + hq) * kPartialFloats + 128]);
        const float* row = cb + tid * kPartialFloats;  // warp tid / 4, head tid % 4
        const float f = exp2f(row[128] - (M == -INFINITY ? 0.f : M));
        wf[tid] = f;
        wl[tid] = row[129] * f;
        if (tid < kGroup) wm[hq] = M;
    }
    named_barrier_sync(1, kConsumerThreads);
    // Thread t < 128 merges head t / 32, dims 4 (t % 32) .. +3.
    float* part = clustered                     ? cpart
                  : (exchange && n_split == 1) ? xrows
                                               : a.ws_partials + ((int64_t)lsplit * kNumKVHeads + h) * kGroup * kPartialFloats;
    if (tid < kOutputs / 4) {
        const int hq = tid >> 5, d0 = (tid & 31) * 4;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float f = wf[w * kGroup + hq];
            const float4 x = *reinterpret_cast<const float4*>(cb + (w * kGroup + hq) * kPartialFloats + d0);
            O = make_float4(fmaf(x.x, f, O.x), fmaf(x.y, f, O.y), fmaf(x.z, f, O.z), fmaf(x.w, f, O.w));
            L += wl[w * kGroup + hq];
        }
        const float M = wm[hq];
        if (n_split == 1 && !clustered && !exchange) {
            write_result4(direct, b, h * kGroup + hq, d0, O, M, L);
        } else {
            float* row = part + hq * kPartialFloats;
            *reinterpret_cast<float4*>(row + d0) = O;
            if (d0 == 0) {
                row[128] = M;
                row[129] = L;
            }
        }
    }
    if (clustered) {
        cluster_merge(a.cluster, gsplit, c, lane, cpart, direct, h);
    } else if (exchange && n_split == 1) {
        named_barrier_sync(1, kConsumerThreads);
        exchange_and_finish(a, h, tid, xrows, info, direct);
    } else if (a.ws_arrivals != nullptr && n_split > 1) {
        last_split_merge(a, n_split, h, tid, lsm, info + 2, direct, xrows, info);
    }
}

// ---------------------------------------------------------------------------
// decode_queue_kernel: the decode of a batch of sequences, one CTA per SM.
// Each CTA's producer warp takes items w = 0, 1, ... in order from a work
// queue in the workspace header, item w being split w / n_heads of the plan,
// of KV head w % n_heads: decode_kernel's CTA order, every sequence's
// full-chunk splits first and the shorter last splits after them.  The
// consumers compute each item exactly as decode_kernel does and store its FP32
// partial (a sequence of one split: its BF16 rows); split_merge_kernel then
// finishes the sequences.  The next item's Q rows and tiles stream into the
// ring while the consumers merge the current one, so an SM does not sit idle
// between splits as it does between the CTAs of a grid of one split per CTA.
// Which CTA computes an item does not change its result.
// ---------------------------------------------------------------------------
template <bool kKRotated>
__global__ void __launch_bounds__(kThreads, 1) decode_queue_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* empty = full + kStages;
    uint64_t* qbar = reinterpret_cast<uint64_t*>(smem + kQueueOffBars);  // [2]: the Q-row slots
    uint64_t* slot_filled = qbar + 2;                                       // [2]: an item slot written
    uint64_t* slot_freed = qbar + 4;                                        // [2]: an item slot read
    int* slots = reinterpret_cast<int*>(smem + kQueueOffItems);            // [2][kItemInts]
    float* pbuf = reinterpret_cast<float*>(smem + kOffP);
    float* abuf = reinterpret_cast<float*>(smem + kOffAlpha);
    float2* rope = reinterpret_cast<float2*>(smem + kOffRope);
    const RopeTable* rt = a.rope;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tid = threadIdx.x;
    const int c = warp;
    const int slot = lane >> 3;  // key within the group of 4 a step handles
    const int g = lane & 7;      // pairs 8g .. 8g+7 (dims 8g..8g+7 and 64+8g..64+8g+7)
    const int hh = g >> 1;       // Q head whose score this lane holds after the reduction

    // ---- set-up that reads only the argument block: before the dependency wait
    if (tid == kConsumerThreads) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kKRotated ? 1 : 2);  // + the producer warp's Q_T
            mbar_init(&empty[s], kConsumerWarps);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&qbar[s], 1);
            mbar_init(&slot_filled[s], 1);
            mbar_init(&slot_freed[s], kConsumerWarps);  // one arrival per consumer warp
        }
        fence_barrier_init();
        prefetch_tensormap(&a.kmap);
        prefetch_tensormap(&a.vmap);
    }
    // RoPE constants, as in decode_kernel.
    float2 qfr[4], qfi[4], kfr[kSteps][4], kfi[kSteps][4];
    ProducerRope prope{};
    if (!kKRotated && warp < kConsumerWarps) {
#pragma unroll
        for (int step = 0; step < kSteps; ++step)
            rope_row8(rt->key_off[c * kKeysPerWarp + step * 4 + slot], g, kfr[step], kfi[step]);
    }
    if (!kKRotated && warp == kConsumerWarps) {
        prope.step0 = rt->step[2 * lane];
        prope.step1 = rt->step[2 * lane + 1];
        const float2 t0 = rt->rot_tile[2 * lane], t1 = rt->rot_tile[2 * lane + 1];
        prope.back_r = make_float2(t0.x, t1.x);
        prope.back_i = make_float2(-t0.y, -t1.y);
    }
    auto lane_rope = [&](int qpos) {
        if (tid < kPairs) rope[kRopeQ * kPairs + tid] = rope_factor(rt->step[tid], qpos);
        named_barrier_sync(1, kConsumerThreads);
        rope_row8(rope + kRopeQ * kPairs, g, qfr, qfi);
        if (a.flags & GQA_FLAG_Q_ROTATED) {  // Q supplied rotated: identity factors (exact)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                qfr[jj] = make_float2(1.f, 1.f);
                qfi[jj] = make_float2(0.f, 0.f);
            }
        }
    };
    __syncthreads();  // the barriers are initialised
    allow_dependent_launch();
    grid_dependency_wait();

    // ======================= producer warp =======================
    if (warp == kConsumerWarps) {
        int ring = 0, issued = 0, rotated = 0, n_q = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int sl = k & 1;
            int w = 0;
            if (lane == 0) w = (int)atomicAdd(a.ws_work, 1u);
            w = __shfl_sync(0xffffffffu, w, 0);
            bool valid = w < a.n_items;
            const int item_split = w / a.n_heads, item_hm = w % a.n_heads;
            // The slot (and its Q rows) of item k - 2 must have been read.
            if (k >= 2) {
                bool w2 = true;
                if (lane == 0) w2 = mbar_wait(&slot_freed[sl], ((k >> 1) - 1) & 1);
                if (!__shfl_sync(0xffffffffu, w2 ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
            }
            int b = 0, split = item_split, logical = item_split;
            if (valid) {
                // Sequence b has full_b = keys / chunk full splits and
                // seq_splits - full_b (0 or 1) shorter last ones.
                auto counts = [&](int bb, int& nf, int& np) {
                    nf = np = 0;
                    if (bb < a.batch) {
                        const SeqDesc db = a.descs[bb];
                        nf = seq_key_count(db) / a.chunk;
                        np = seq_splits(db, a.chunk) - nf;
                    }
                };
                auto scan = [&](int v) {
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int t = __shfl_up_sync(0xffffffffu, v, o);
                        if (lane >= o) v += t;
                    }
                    return v;
                };
                int total_full = 0;
                for (int b0 = 0; b0 < a.batch; b0 += 32) {
                    int nf, np;
                    counts(b0 + lane, nf, np);
                    total_full += __shfl_sync(0xffffffffu, scan(nf), 31);
                }
                const bool in_full = item_split < total_full;
                const int target = in_full ? item_split : item_split - total_full;
                int base = 0, sbase = 0;  // splits of the chosen kind / of any kind before b0
                b = -1;
                for (int b0 = 0; b0 < a.batch && b < 0; b0 += 32) {
                    int nf, np;
                    counts(b0 + lane, nf, np);
                    const int nk = in_full ? nf : np;
                    const int incl = scan(nk), sincl = scan(nf + np);
                    const int excl = incl - nk;
                    const bool hit = b0 + lane < a.batch && target >= base + excl && target < base + incl;
                    const unsigned m = __ballot_sync(0xffffffffu, hit);
                    if (m) {
                        const int src = __ffs(m) - 1;
                        b = b0 + src;
                        const int nf_src = __shfl_sync(0xffffffffu, nf, src);
                        split = in_full ? target - base - __shfl_sync(0xffffffffu, excl, src) : nf_src;
                        const int sexcl = __shfl_sync(0xffffffffu, sincl - (nf + np), src);
                        logical = sbase + sexcl + split;
                    }
                    base += __shfl_sync(0xffffffffu, incl, 31);
                    sbase += __shfl_sync(0xffffffffu, sincl, 31);
                }
                valid = b >= 0;
            }
            SeqDesc d = a.single;
            if (valid) d = a.descs[b];
            const int key0 = split * a.chunk;
            const int cnt = max(0, min(a.chunk, seq_key_count(d) - key0));
            if (lane == 0) {  // everything the consumers need to know about the item
                int* it = slots + sl * kItemInts;
                it[0] = valid ? 1 : 0;
                it[1] = b;
                it[2] = split;
                it[3] = logical;
                it[4] = item_hm;
                it[5] = seq_splits(d, a.chunk);
                it[6] = cnt;
                it[7] = d.query_position;
                it[8] = d.seq_len;
                mbar_arrive(&slot_filled[sl]);
            }
            if (!valid) break;
            const int n_tiles = (cnt + kTileKeys - 1) / kTileKeys;
            // m - T of the item's first tile (Q supplied rotated: m = 0).
            const int64_t q_minus_first =
                ((a.flags & GQA_FLAG_Q_ROTATED) ? 0 : (int64_t)d.query_position) - ((int64_t)d.pos_begin + key0);
            ok = produce_item<kKRotated>(a, smem, full, empty, &qbar[sl], (uint32_t)((k >> 1) & 1),
                                         smem + kQueueOffQ + sl * kGroup * kRowBytes, b, a.head0 + item_hm,
                                         item_hm, d.kv_start + key0, n_tiles, q_minus_first, prope, lane, ring,
                                         issued, rotated);
            n_q = k + 1;
            ring += n_tiles;
        }
        if (lane == 0) {
            if (!ok) atomicOr(a.ws_status, kDevStatusTimeout);
            // Do not leave while copies into this CTA's shared memory are in
            // flight (after a failed wait, complete the stages whose Q_T was
            // not written).
            if (!kKRotated)
                for (int p = rotated; p < issued; ++p) mbar_arrive(&full[p % kStages]);
            for (int p = max(0, issued - kStages); p < issued; ++p) mbar_wait(&full[p % kStages], (p / kStages) & 1);
            for (int k = max(0, n_q - 2); k < n_q; ++k) mbar_wait(&qbar[k & 1], (k >> 1) & 1);
            // The last CTA to leave the queue clears it for the next call (which
            // starts after this grid completes).
            if (arrive_acq_rel_gpu(a.ws_work + 1) == gridDim.x - 1) {
                a.ws_work[0] = 0u;
                a.ws_work[1] = 0u;
            }
        }
        return;
    }

    // ======================= consumer warps =======================
    float* pw = pbuf + c * 2 * (kKeysPerWarp * kGroup);  // this warp's probabilities [2][keys][4 heads]
    float* aw = abuf + c * 2 * kGroup;                    // and rescales [2][4]
    float* cb = reinterpret_cast<float*>(smem + kQueueOffEpi);
    float* wf = cb + kConsumerWarps * kGroup * kPartialFloats;  // [w][hq]  2^(m_w - M)
    float* wl = wf + kConsumerWarps * kGroup;                   // [w][hq]  l_w * 2^(m_w - M)
    float* wm = wl + kConsumerWarps * kGroup;                   // [hq]     M
    const OutSpec direct{a.out, a.o_bstride, a.o_hstride, a.flags};
    bool ok = true;
    int ring0 = 0;  // ring position of the item's first tile
    for (int k = 0;; ++k) {
        const int sl = k & 1;
        // Every consumer warp runs the same items: a wait that timed out in one
        // of them stops all of them here (named barriers do not time out).
        const bool filled = mbar_wait(&slot_filled[sl], (k >> 1) & 1);
        if (named_barrier_or(1, kConsumerThreads, !filled)) {
            ok = false;
            break;
        }
        const int* it = slots + sl * kItemInts;
        if (it[0] == 0) break;
        const int b = it[1];
        const int split = it[2];
        const int lsplit = it[3];  // storage index of this split's partial
        const int hm = it[4];
        const int h = a.head0 + hm;
        const int n_split = it[5];
        const int cnt = it[6];
        const int qpos = it[7];
        const int seq_len = it[8];
        const int n_tiles = (cnt + kTileKeys - 1) / kTileKeys;

        // Q pre-scaled by scale*log2(e): rotated at QUERY_POSITION once per item
        // (K pre-rotated), or to each tile's first key by the producer (loaded
        // per tile in qk_tile).  Register slot j of a lane holds Q head j ^ hh.
        float2 qr[kGroup][4], qi[kGroup][4];
        if constexpr (kKRotated) {
            lane_rope(qpos);
            ok = mbar_wait(&qbar[sl], (k >> 1) & 1);
            const uint8_t* qs = smem + kQueueOffQ + sl * kGroup * kRowBytes;
#pragma unroll
            for (int j = 0; j < kGroup; ++j) {
                const uint8_t* qrow = qs + (j ^ hh) * kRowBytes;
                const uint4 xr = *reinterpret_cast<const uint4*>(qrow + g * 16);
                const uint4 xi = *reinterpret_cast<const uint4*>(qrow + 128 + g * 16);
                const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
                const uint32_t yw[4] = {xi.x, xi.y, xi.z, xi.w};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    float2 re, im;
                    cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), qfr[jj], qfi[jj], re, im);
                    qr[j][jj] = __fmul2_rn(re, f2(a.qscale));
                    qi[j][jj] = __fmul2_rn(im, f2(a.qscale));
                }
            }
        }
        // The slot (and its Q rows) may be reused.
        __syncwarp();
        if (lane == 0) mbar_arrive(&slot_freed[sl]);

        // The split merge finds each sequence's splits here.
        if (split == 0 && hm == 0 && tid == 0 && n_split > 1) a.ws_seqinfo[b] = make_int2(lsplit, n_split);
        if (a.mask_out != nullptr && split == 0 && hm == 0) {
            const int n_pad = ((seq_len + a.kv_block_len - 1) / a.kv_block_len) * a.kv_block_len;
            for (int p = tid; p < n_pad; p += kConsumerThreads)
                a.mask_out[(int64_t)b * a.mask_stride + p] = key_valid(p, seq_len, qpos) ? 1 : 0;
        }

        float m_run = -INFINITY;  // running max (log2 units) of head hh
        float l_run = 0.f;        // running sum of this lane's key slot for head hh
        float2 acc0[kGroup], acc1[kGroup];  // dims (4*lane, +1) and (4*lane+2, +3) of each head
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq) acc0[hq] = acc1[hq] = make_float2(0.f, 0.f);

        // Scores of this warp's keys of tile t: RoPE of K, Q.K for the 4 heads,
        // reduction over the 8 lanes of each key.  Keys [key0, key0 + cnt) all
        // satisfy key_valid() (they lie in [0, min(SEQ_LEN, QUERY_POSITION + 1)));
        // rows past them are masked.
        auto qk_tile = [&](int t, float (&sc)[kSteps]) {
            const uint8_t* kt = smem + ((ring0 + t) % kStages) * kStageBytes;
            const int rows = min(kTileKeys, cnt - t * kTileKeys);
            if constexpr (!kKRotated) {
                const float* qt = reinterpret_cast<const float*>(smem + kOffQt) + ((ring0 + t) % kStages) * kQtFloats;
#pragma unroll
                for (int j = 0; j < kGroup; ++j) {
                    const float* row = qt + (j ^ hh) * kHeadDim + 4 * g;
                    const float4 r0 = *reinterpret_cast<const float4*>(row);
                    const float4 r1 = *reinterpret_cast<const float4*>(row + 32);
                    const float4 i0 = *reinterpret_cast<const float4*>(row + 64);
                    const float4 i1 = *reinterpret_cast<const float4*>(row + 96);
                    qr[j][0] = make_float2(r0.x, r0.y);
                    qr[j][1] = make_float2(r0.z, r0.w);
                    qr[j][2] = make_float2(r1.x, r1.y);
                    qr[j][3] = make_float2(r1.z, r1.w);
                    qi[j][0] = make_float2(i0.x, i0.y);
                    qi[j][1] = make_float2(i0.z, i0.w);
                    qi[j][2] = make_float2(i1.x, i1.y);
                    qi[j][3] = make_float2(i1.z, i1.w);
                }
            }
#pragma unroll
            for (int step = 0; step < kSteps; ++step) {
                const int r = c * kKeysPerWarp + step * 4 + slot;
                const uint4 kre = *reinterpret_cast<const uint4*>(kt + r * kRowBytes + g * 16);
                const uint4 kim = *reinterpret_cast<const uint4*>(kt + r * kRowBytes + 128 + g * 16);
                const uint32_t xw[4] = {kre.x, kre.y, kre.z, kre.w};
                const uint32_t yw[4] = {kim.x, kim.y, kim.z, kim.w};
                float2 rr[4], ri[4];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    if constexpr (kKRotated) {
                        rr[jj] = bf16x2_to_float2(xw[jj]);
                        ri[jj] = bf16x2_to_float2(yw[jj]);
                    } else {
                        cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), kfr[step][jj], kfi[step][jj], rr[jj],
                              ri[jj]);
                    }
                }
                float s[kGroup];
#pragma unroll
                for (int hq = 0; hq < kGroup; ++hq) {
                    float2 acc = __fmul2_rn(qr[hq][0], rr[0]);
                    acc = __ffma2_rn(qi[hq][0], ri[0], acc);
#pragma unroll
                    for (int jj = 1; jj < 4; ++jj) {
                        acc = __ffma2_rn(qr[hq][jj], rr[jj], acc);
                        acc = __ffma2_rn(qi[hq][jj], ri[jj], acc);
                    }
                    s[hq] = acc.x + acc.y;
                }
                // Lanes l and l^4 hold the same heads in swapped slot pairs, lanes l
                // and l^2 in swapped slots: keep 0/1, send 2/3; keep 0, send 1.
                const float t0 = s[0] + __shfl_xor_sync(0xffffffffu, s[2], 4);
                const float t1 = s[1] + __shfl_xor_sync(0xffffffffu, s[3], 4);
                float u = t0 + __shfl_xor_sync(0xffffffffu, t1, 2);
                u += __shfl_xor_sync(0xffffffffu, u, 1);
                sc[step] = r < rows ? u : -INFINITY;
            }
        };

        // Online softmax of head hh over this warp's keys of one tile, in
        // registers: the probabilities pv and the rescale alpha of the running sums.
        auto softmax_tile = [&](const float (&sc)[kSteps], float (&pv)[kSteps], float& alpha) {
            float mx = sc[0];
#pragma unroll
            for (int step = 1; step < kSteps; ++step) mx = fmaxf(mx, sc[step]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float m_new = fmaxf(m_run, mx);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            alpha = fast_exp2(m_run - m_use);
            float psum = 0.f;
#pragma unroll
            for (int step = 0; step < kSteps; ++step) {
                pv[step] = fast_exp2(sc[step] - m_use);
                psum += pv[step];
            }
            l_run = l_run * alpha + psum;
            m_run = m_new;
        };
        // Stores p and the rescale into the warp's buffer `buf`; the caller's
        // __syncwarp publishes them to the warp.
        auto publish = [&](const float (&pv)[kSteps], float alpha, int buf) {
            float* pb = pw + buf * (kKeysPerWarp * kGroup);
            if ((g & 1) == 0) {
#pragma unroll
                for (int step = 0; step < kSteps; ++step) pb[(step * 4 + slot) * kGroup + hh] = pv[step];
                if (slot == 0) aw[buf * kGroup + hh] = alpha;
            }
        };

        // acc = acc * alpha + sum_k p_k * V_k over this warp's keys of tile t.
        // In the split's last tile, rows past its keys may hold anything (even
        // NaN): their probabilities are 0, and each lane zeroes the 8 bytes of
        // those rows that it reads itself, so no other lane is involved.
        auto pv_tile = [&](int t, int buf, bool last) {
            uint8_t* vt = smem + ((ring0 + t) % kStages) * kStageBytes + kTileBytes;
            if (last) {
                const int nr = min(kTileKeys, cnt - t * kTileKeys) - c * kKeysPerWarp;
#pragma unroll
                for (int rr = 0; rr < kKeysPerWarp; ++rr)
                    if (rr >= nr)
                        *reinterpret_cast<uint2*>(vt + (c * kKeysPerWarp + rr) * kRowBytes + lane * 8) = make_uint2(0u, 0u);
            }
            const float* pb = pw + buf * (kKeysPerWarp * kGroup);
            const float4 al = *reinterpret_cast<const float4*>(aw + buf * kGroup);
            const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq) {
                acc0[hq] = __fmul2_rn(acc0[hq], f2(alv[hq]));
                acc1[hq] = __fmul2_rn(acc1[hq], f2(alv[hq]));
            }
#pragma unroll
            for (int rr = 0; rr < kKeysPerWarp; ++rr) {
                const float4 p4 = *reinterpret_cast<const float4*>(pb + rr * kGroup);
                const uint2 vv = *reinterpret_cast<const uint2*>(vt + (c * kKeysPerWarp + rr) * kRowBytes + lane * 8);
                const float2 v0 = bf16x2_to_float2(vv.x), v1 = bf16x2_to_float2(vv.y);
                const float pk[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                for (int hq = 0; hq < kGroup; ++hq) {
                    acc0[hq] = ffma2_bcast(pk[hq], v0, acc0[hq]);
                    acc1[hq] = ffma2_bcast(pk[hq], v1, acc1[hq]);
                }
            }
        };

        // Software pipeline: one iteration computes the scores and the softmax of
        // tile t and the P.V of tile t-1, with no branch or warp barrier between
        // them, so that the two independent instruction streams interleave; the
        // probabilities of tile t are stored after the P.V loads of tile t-1 (a
        // different buffer) and published by one __syncwarp.
        if (ok && n_tiles > 0) {
            if (mbar_wait(&full[ring0 % kStages], (ring0 / kStages) & 1)) {
                float sc[kSteps], pv[kSteps], alpha;
                qk_tile(0, sc);
                softmax_tile(sc, pv, alpha);
                publish(pv, alpha, 0);
                __syncwarp();
            } else {
                ok = false;
            }
        }
        for (int t = 1; t < n_tiles && ok; ++t) {
            if (!mbar_wait(&full[(ring0 + t) % kStages], ((ring0 + t) / kStages) & 1)) {
                ok = false;
                break;
            }
            float sc[kSteps], pv[kSteps], alpha;
            qk_tile(t, sc);
            softmax_tile(sc, pv, alpha);
            pv_tile(t - 1, (t - 1) & 1, false);
            publish(pv, alpha, t & 1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[(ring0 + t - 1) % kStages]);
        }
        if (ok && n_tiles > 0) {
            pv_tile(n_tiles - 1, (n_tiles - 1) & 1, true);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[(ring0 + n_tiles - 1) % kStages]);
        }
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);

        // ---- merge the warps through the epilogue region, once every consumer
        // has finished the previous item's epilogue; a timed-out wait in any
        // warp ends the item loop after this item, for all of them.
        const bool any_failed = named_barrier_or(1, kConsumerThreads, !ok);
        {
            float* mine = cb + c * kGroup * kPartialFloats;
#pragma unroll
            for (int hq = 0; hq < kGroup; ++hq)
                *reinterpret_cast<float4*>(mine + hq * kPartialFloats + 4 * lane) =
                    make_float4(acc0[hq].x, acc0[hq].y, acc1[hq].x, acc1[hq].y);
            if (slot == 0 && (g & 1) == 0) {
                mine[hh * kPartialFloats + 128] = m_run;
                mine[hh * kPartialFloats + 129] = l_run;
            }
        }
        named_barrier_sync(1, kConsumerThreads);
        // Factors once per (warp, head): thread t < 44 owns warp t / 4, head t % 4.
        if (tid < kConsumerWarps * kGroup) {
            const int hq = tid & 3;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cb[(w * kGroup + hq) * kPartialFloats + 128]);
            const float* row = cb + tid * kPartialFloats;  // warp tid / 4, head tid % 4
            const float f = exp2f(row[128] - (M == -INFINITY ? 0.f : M));
            wf[tid] = f;
            wl[tid] = row[129] * f;
            if (tid < kGroup) wm[hq] = M;
        }
        named_barrier_sync(1, kConsumerThreads);
        // Thread t < 128 merges head t / 32, dims 4 (t % 32) .. +3.
        if (tid < kOutputs / 4) {
            const int hq = tid >> 5, d0 = (tid & 31) * 4;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
            float L = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float f = wf[w * kGroup + hq];
                const float4 x = *reinterpret_cast<const float4*>(cb + (w * kGroup + hq) * kPartialFloats + d0);
                O = make_float4(fmaf(x.x, f, O.x), fmaf(x.y, f, O.y), fmaf(x.z, f, O.z), fmaf(x.w, f, O.w));
                L += wl[w * kGroup + hq];
            }
            const float M = wm[hq];
            if (n_split == 1) {
                write_result4(direct, b, h * kGroup + hq, d0, O, M, L);
            } else {
                float* row = a.ws_partials + ((int64_t)lsplit * kNumKVHeads + h) * kGroup * kPartialFloats +
                             hq * kPartialFloats;
                *reinterpret_cast<float4*>(row + d0) = O;
                if (d0 == 0) {
                    row[128] = M;
                    row[129] = L;
                }
            }
        }
        ring0 += n_tiles;
        if (any_failed) {
            ok = false;
            break;
        }
    }
    if (!ok && lane == 0) atomicOr(a.ws_status, kDevStatusTimeout);
}

// ---------------------------------------------------------------------------
// Merge of a sequence's split partials: one CTA per (sequence, Q head), one
// thread per dim.  Runs after decode_kernel (griddepcontrol.wait).
// ---------------------------------------------------------------------------
struct MergeArgs {
    const float* partials;  // [total_splits][32][132]
    const int2* seqinfo;    // [batch]: (first global split, splits) of sequences with > 1 split
    const SeqDesc* descs;   // nullptr: single sequence, splits from `single_splits`
    int single_splits;
    int chunk;
    OutSpec out;
    int qh0, n_qh;          // the call's Q heads [qh0, qh0 + n_qh)
};

__global__ void __launch_bounds__(kHeadDim) split_merge_kernel(const __grid_constant__ MergeArgs m) {
    __shared__ float fac[kMaxSplitsPerSeq];
    __shared__ float red[2][4];
    allow_dependent_launch();
    const int b = blockIdx.x / m.n_qh;
    const int qh = m.qh0 + (int)(blockIdx.x % m.n_qh);
    const int dim = threadIdx.x;
    grid_dependency_wait();
    const int n_split = m.descs == nullptr ? m.single_splits : seq_splits(m.descs[b], m.chunk);
    if (n_split <= 1) return;  // written directly by decode_kernel
    const int2 si = m.seqinfo[b];
    const int64_t split_stride = (int64_t)kNumQHeads * kPartialFloats;
    const float* base = m.partials + ((int64_t)si.x * kNumQHeads + qh) * kPartialFloats;
    // One round trip: split s's (m, l) on thread s, and this thread's acc column
    // of the first 32 splits, all loaded before any of them is used.
    float ms = -INFINITY, ls = 0.f;
    if (dim < n_split) {
        ms = __ldcg(base + dim * split_stride + 128);
        ls = __ldcg(base + dim * split_stride + 129);
    }
    constexpr int kBatch = 32;
    float v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) v[j] = j < n_split ? __ldcg(base + j * split_stride + dim) : 0.f;
    float M = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if ((dim & 31) == 0) red[0][dim >> 5] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
    const float Mu = M == -INFINITY ? 0.f : M;
    const float f = dim < n_split ? exp2f(ms - Mu) : 0.f;
    if (dim < n_split) fac[dim] = f;
    float L = ls * f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if ((dim & 31) == 0) red[1][dim >> 5] = L;
    __syncthreads();
    L = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
    float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kBatch; ++j) o4[j & 3] = fmaf(v[j], j < n_split ? fac[j] : 0.f, o4[j & 3]);
    for (int s = kBatch; s < n_split; ++s) o4[s & 3] = fmaf(__ldcg(base + s * split_stride + dim), fac[s], o4[s & 3]);
    const float O = (o4[0] + o4[1]) + (o4[2] + o4[3]);
    write_result(m.out, b, qh, dim, O, M, L);
}

// ---------------------------------------------------------------------------
// Cross-shard combine: one CTA per (sequence, Q head), one thread per dim.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) combine_kernel(const float* __restrict__ parts, int n_parts,
                                                      int64_t part_stride, int64_t batch_stride,
                                                      __nv_bfloat16* __restrict__ out, int64_t o_bstride,
                                                      int64_t o_hstride) {
    const int b = blockIdx.x / kNumQHeads;
    const int qh = blockIdx.x % kNumQHeads;
    const int dim = threadIdx.x;
    const float* base = parts + (int64_t)b * batch_stride + (int64_t)qh * kPartialFloats;
    float M = -INFINITY;
    for (int s = 0; s < n_parts; ++s) M = fmaxf(M, base[(int64_t)s * part_stride + 128]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
    for (int s = 0; s < n_parts; ++s) {
        const float* row = base + (int64_t)s * part_stride;
        const float f = exp2f(row[128] - Mu);
        L = fmaf(row[129], f, L);
        O = fmaf(row[dim], f, O);
    }
    out[(int64_t)b * o_bstride + (int64_t)qh * o_hstride + dim] = __float2bfloat16_rn(O / L);
}

// ---------------------------------------------------------------------------
// RoPE of whole rows (one warp per row; lane owns pairs 2*lane, 2*lane+1).
// ---------------------------------------------------------------------------
struct RopeSteps {
    uint64_t step[kPairs];
};

__global__ void __launch_bounds__(256) rope_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const int32_t* __restrict__ pos, float* __restrict__ out,
                                                        int rows, const __grid_constant__ RopeSteps steps) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t p = pos[row];
    const __nv_bfloat16* xr = x + (int64_t)row * kHeadDim;
    float* o = out + (int64_t)row * kHeadDim;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int i = 2 * lane + j;
        const float2 f = rope_factor(steps.step[i], p);
        const float xv = __bfloat162float(xr[i]), yv = __bfloat162float(xr[i + kPairs]);
        o[i] = xv * f.x - yv * f.y;
        o[i + kPairs] = xv * f.y + yv * f.x;
    }
}

// Pre-rotated K cache: one warp per (position, KV head) row, lane l owns pairs
// 2l and 2l+1 (elements i, i+64), exact factors per element, BF16 out (RNE).
// In place is safe: every element is read and written by the same lane.
__global__ void __launch_bounds__(256) rope_k_cache_kernel(const __nv_bfloat16* k, __nv_bfloat16* out,
                                                           const int32_t* __restrict__ pos, int rows,
                                                           int64_t pos_stride, int64_t head_stride,
                                                           const __grid_constant__ RopeSteps steps) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int i_pos = row / kNumKVHeads, h = row % kNumKVHeads;
    const int64_t p = pos[i_pos];
    const int64_t off = (int64_t)i_pos * pos_stride + (int64_t)h * head_stride;
    const int i = 2 * lane;
    const __nv_bfloat162 x2 = *reinterpret_cast<const __nv_bfloat162*>(k + off + i);
    const __nv_bfloat162 y2 = *reinterpret_cast<const __nv_bfloat162*>(k + off + i + kPairs);
    const float2 xv = __bfloat1622float2(x2), yv = __bfloat1622float2(y2);
    const float2 f0 = rope_factor(steps.step[i], p), f1 = rope_factor(steps.step[i + 1], p);
    const float re0 = fmaf(xv.x, f0.x, -(yv.x * f0.y)), im0 = fmaf(xv.x, f0.y, yv.x * f0.x);
    const float re1 = fmaf(xv.y, f1.x, -(yv.y * f1.y)), im1 = fmaf(xv.y, f1.y, yv.y * f1.x);
    *reinterpret_cast<__nv_bfloat162*>(out + off + i) = __floats2bfloat162_rn(re0, re1);
    *reinterpret_cast<__nv_bfloat162*>(out + off + i + kPairs) = __floats2bfloat162_rn(im0, im1);
}

// Launch with programmatic dependent launch and, for cluster_x > 0, thread-block
// clusters of (cluster_x, 1, 1).
cudaError_t launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args,
                       int cluster_x = 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cluster_x > 0) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = cluster_x;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelExC(&cfg, func, args);
}

// Immutable RoPE tables, one slot per distinct rope_theta (per device).
__device__ RopeTable g_rope_tables[kRopeTableSlots];

}  // namespace

// Host side of the RoPE table cache.
namespace {
struct RopeSlots {
    bool used[kRopeTableSlots] = {};
    double theta[kRopeTableSlots] = {};
};
std::mutex g_rope_mu;
RopeSlots g_rope_slots[64];

void build_rope_table_host(double theta, RopeTable& t) {
    const double two_pi = 2.0 * M_PI;
    for (int i = 0; i < kPairs; ++i) {
        const double inv = std::pow(theta, -2.0 * i / (double)kHeadDim);
        t.step[i] = (uint64_t)std::llround(inv / two_pi * 18446744073709551616.0);  // < 2^62
        t.rot_tile[i] = make_float2((float)std::cos(kTileKeys * inv), (float)std::sin(kTileKeys * inv));
        for (int r = 0; r < kTileKeys; ++r)
            t.key_off[r][i] = make_float2((float)std::cos(r * inv), (float)std::sin(r * inv));
    }
}
}  // namespace

cudaError_t rope_table_for(double theta, const RopeTable** table, bool* out_of_slots) {
    *out_of_slots = false;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_rope_mu);
    RopeSlots& rs = g_rope_slots[dev];
    int slot = -1;
    for (int i = 0; i < kRopeTableSlots && slot < 0; ++i)
        if (rs.used[i] && rs.theta[i] == theta) slot = i;
    void* base = nullptr;
    e = cudaGetSymbolAddress(&base, g_rope_tables);
    if (e != cudaSuccess) return e;
    if (slot < 0) {
        for (int i = 0; i < kRopeTableSlots && slot < 0; ++i)
            if (!rs.used[i]) slot = i;
        if (slot < 0) {
            *out_of_slots = true;
            return cudaSuccess;
        }
        RopeTable host;
        build_rope_table_host(theta, host);
        e = cudaMemcpy(static_cast<RopeTable*>(base) + slot, &host, sizeof(RopeTable), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        rs.used[slot] = true;
        rs.theta[slot] = theta;
    }
    *table = static_cast<const RopeTable*>(base) + slot;
    return cudaSuccess;
}

int decode_tile_keys() { return kTileKeys; }
int decode_max_splits() { return kMaxSplitsPerSeq; }
size_t decode_smem_bytes() { return kSmemBytes; }

int decode_max_cluster_splits() { return kMaxClusterSplits; }
int decode_last_merge_max_splits() { return kLastMergeMaxSplits; }

cudaError_t decode_prepare(int device) {
    (void)device;
    for (const void* f : {reinterpret_cast<const void*>(decode_kernel<false>),
                          reinterpret_cast<const void*>(decode_kernel<true>)}) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        // Clusters of up to 16 CTAs (above 8 is opt-in); without it clusters stay off.
        if (cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            (void)cudaGetLastError();
    }
    for (const void* f : {reinterpret_cast<const void*>(decode_queue_kernel<false>),
                          reinterpret_cast<const void*>(decode_queue_kernel<true>)}) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kQueueSmemBytes);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int decode_cluster_capacity(int cluster) {
    if (cluster < 2 || cluster > kMaxClusterSplits) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster, kNumKVHeads);  // the occupancy query counts clusters, whatever the grid
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, decode_kernel<false>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_decode(const DecodeArgs& a, int total_splits, cudaStream_t stream) {
    void* dargs[] = {const_cast<DecodeArgs*>(&a)};
    const void* kern = (a.flags & GQA_FLAG_K_ROTATED) ? reinterpret_cast<const void*>(decode_kernel<true>)
                                                       : reinterpret_cast<const void*>(decode_kernel<false>);
    cudaError_t e;
    if (a.cluster > 0) {  // single sequence, merged inside the clusters
        return launch_pdl(kern, dim3(a.cluster, a.n_heads), dim3(kThreads), kSmemBytes, stream, dargs, a.cluster);
    } else if (a.ws_work != nullptr) {  // a batch: one CTA per SM works through the items
        int dev = 0, sms = 0;
        e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        const void* qk = (a.flags & GQA_FLAG_K_ROTATED) ? reinterpret_cast<const void*>(decode_queue_kernel<true>)
                                                         : reinterpret_cast<const void*>(decode_queue_kernel<false>);
        e = launch_pdl(qk, dim3(std::min(a.n_items, sms)), dim3(kThreads), kQueueSmemBytes, stream, dargs);
    } else {
        e = launch_pdl(kern, dim3(total_splits * a.n_heads), dim3(kThreads), kSmemBytes, stream, dargs);
    }
    // Done when every sequence had one split or the last split of each head merged.
    if (e != cudaSuccess || total_splits <= a.batch || a.ws_arrivals != nullptr) return e;
    MergeArgs m;
    m.partials = a.ws_partials;
    m.seqinfo = a.ws_seqinfo;
    m.descs = a.descs;
    m.single_splits = a.descs == nullptr ? total_splits : 0;
    m.chunk = a.chunk;
    m.out = OutSpec{a.out, a.o_bstride, a.o_hstride, a.flags};
    m.qh0 = a.head0 * kGroup;
    m.n_qh = a.n_heads * kGroup;
    void* margs[] = {&m};
    return launch_pdl(reinterpret_cast<const void*>(split_merge_kernel), dim3(a.batch * m.n_qh), dim3(kHeadDim), 0,
                      stream, margs);
}

cudaError_t launch_combine(const float* parts, int n_parts, int64_t part_stride, int64_t batch_stride, int batch,
                           void* out, int64_t o_bstride, int64_t o_hstride, cudaStream_t stream) {
    combine_kernel<<<batch * kNumQHeads, kHeadDim, 0, stream>>>(
        parts, n_parts, part_stride, batch_stride, static_cast<__nv_bfloat16*>(out), o_bstride, o_hstride);
    return cudaGetLastError();
}

cudaError_t launch_rope_rows(const void* x, const int32_t* pos, float* out, int rows, const uint64_t* step,
                             cudaStream_t stream) {
    RopeSteps s;
    for (int i = 0; i < kPairs; ++i) s.step[i] = step[i];
    rope_rows_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), pos, out, rows, s);
    return cudaGetLastError();
}

cudaError_t launch_rope_k_cache(const void* k, void* out, const int32_t* pos, int n_positions, int64_t pos_stride,
                                int64_t head_stride, const uint64_t* step, cudaStream_t stream) {
    RopeSteps s;
    for (int i = 0; i < kPairs; ++i) s.step[i] = step[i];
    const int64_t rows = (int64_t)n_positions * kNumKVHeads;
    if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    rope_k_cache_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(out), pos, (int)rows, pos_stride,
        head_stride, s);
    return cudaGetLastError();
}

}  // namespace gqa
