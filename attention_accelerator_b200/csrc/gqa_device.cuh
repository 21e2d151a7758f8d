// gqa_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// geometry constants, the kernel argument block, mbarrier / bulk-copy PTX
// wrappers with bounded waits, BF16 unpacking and the RoPE phase generator.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gqa {

// Llama-3-8B GQA geometry the reference RTL is fixed to
// (gqa_attention_wrapper.v:47-68, axi_lite_regs.v:108-117).
constexpr int kHeadDim = 128;
constexpr int kPairs = kHeadDim / 2;   // rotate_half pairs (i, i+64)
constexpr int kNumQHeads = 32;
constexpr int kNumKVHeads = 8;
constexpr int kGroup = kNumQHeads / kNumKVHeads;
constexpr int kRowBytes = kHeadDim * 2;  // one BF16 K or V row
constexpr int kPartialFloats = 132;      // gqa_partial_row: acc[128], m, l, pad[2]

// Device status word values (first word of the workspace).
constexpr uint32_t kDevStatusTimeout = 1u;

// A bounded wait gives up after this many SM clock cycles (~1 s at 1.9 GHz).
constexpr long long kWaitTimeoutCycles = 2000000000LL;

struct SeqDesc {  // layout-identical to gqa_seq_desc
    int64_t kv_start;
    int32_t seq_len;
    int32_t query_position;
    int32_t pos_begin;
    int32_t pos_end;
};

// Keys a call reads for one sequence: [pos_begin, min(pos_end, n_vis)) with
// n_vis = min(seq_len, query_position + 1), i.e. the positions the hardware
// mask (gqa_attention_wrapper.v:279) lets through.
__host__ __device__ inline int seq_key_begin(const SeqDesc& d) { return d.pos_begin; }
__host__ __device__ inline int seq_key_count(const SeqDesc& d) {
    int n_vis = d.seq_len < d.query_position + 1 ? d.seq_len : d.query_position + 1;
    int hi = d.pos_end < n_vis ? d.pos_end : n_vis;
    int n = hi - d.pos_begin;
    return n > 0 ? n : 0;
}
__host__ __device__ inline int seq_splits(const SeqDesc& d, int chunk) {
    int n = seq_key_count(d);
    int s = (n + chunk - 1) / chunk;
    return s > 0 ? s : 1;
}

// key_valid of gqa_attention_wrapper.v:279 / score_tag_fifo push_key_valid.
__host__ __device__ inline bool key_valid(int64_t p, int seq_len, int query_position) {
    return p < seq_len && p <= query_position;
}

// Decode tiling, shared by the kernel and the host code that builds its tables:
// 11 consumer warps x 8 keys = one 88-key pipeline tile.
constexpr int kDecodeConsumerWarps = 11;
constexpr int kDecodeKeysPerWarp = 8;
constexpr int kDecodeTileKeys = kDecodeConsumerWarps * kDecodeKeysPerWarp;
// Immutable per-(device, rope_theta) RoPE table, computed on the host in double
// precision and uploaded once.  Pair i turns theta^(-2i/128)/(2*pi) turns per
// position; `step` holds that as an unsigned Q0.64 fraction.
struct RopeTable {
    uint64_t step[kPairs];
    float2 rot_tile[kPairs];                  // e^{i theta_i * kDecodeTileKeys}: one tile further
    float2 key_off[kDecodeTileKeys][kPairs];  // e^{i theta_i * r}: key r of a tile relative to its first key
};

// Kernel argument block, passed by value as a __grid_constant__ parameter.  The
// two tensor maps come first: TMA requires them 64-byte aligned in param space.
struct alignas(64) DecodeArgs {
    CUtensorMap kmap;       // K rows: 3-D (dim, row, head) or (dim, head, row), box = one tile of one head
    CUtensorMap vmap;
    int kv_rows_inner;      // 1: rows are tensor-map dimension 1 (head-major), 0: dimension 2
    const __nv_bfloat16* q;
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    void* out;
    int64_t q_bstride, q_hstride;
    int64_t k_pstride, k_hstride;
    int64_t v_pstride, v_hstride;
    int64_t o_bstride, o_hstride;
    const SeqDesc* descs;   // device array, or nullptr: use `single`
    SeqDesc single;
    int batch;
    int chunk;              // keys per split
    float qscale;           // scale * log2(e): scores are kept in log2 units
    uint32_t flags;         // GQA_FLAG_*
    uint32_t* ws_status;
    int2* ws_seqinfo;       // [batch]: (first global split, splits) of sequences with > 1 split
    float* ws_partials;     // [total_splits][8][4][132]
    uint8_t* mask_out;
    int64_t mask_stride;
    int kv_block_len;
    const RopeTable* rope;  // device copy for this call's rope_theta
    int cluster;            // > 0: single sequence, grid (cluster, 8), the splits of a KV head form one
                            // thread-block cluster and merge through distributed shared memory
    uint32_t* ws_arrivals;  // non-null: single sequence, the last split of each KV head to finish merges
                            // (one arrival counter per KV head, zero between calls)
    const uint64_t* peer_bases;  // world > 1: this GPU decodes a shard of one sequence and exchanges the
    int world, rank;             // merged rows with the other ranks' exchange buffers (device array)
    int head0, n_heads;     // KV heads [head0, head0 + n_heads) only; the K/V maps then hold just those
                            // heads (map head index = h - head0).  0 and 8 for a whole call.
    uint32_t* ws_work;      // non-null: a batch run by decode_queue_kernel, one CTA per SM taking the
    int n_items;            // n_items (split, KV head) items from this queue (next item, CTAs done;
                            // both zero between calls)
};

// Exchange buffer of the long-context split (one per rank, mapped by the others):
//   [0] u32 epoch, [4] u32 arrivals, [64] u32 flag[batch * 32], then
//   float rows[2][batch * 32][132] from peer_data_offset(batch), double-buffered by epoch
//   parity: the pull exchange of gqa_combine_peers (each rank publishes into its own buffer);
//   then, from peer_push_offset(batch), the push exchange of the fused decode (one sequence):
//   256 bytes (kPushFlagsBytes, unused by the word protocol) and u64 push_rows[2][kMaxPeers][32][130],
//   each word (epoch << 32 | value bits), which the ranks write into each other's buffers.
constexpr int kPeerFlagsOffset = 64;
constexpr int kMaxPeers = 8;
__host__ __device__ inline size_t peer_data_offset(int batch) {
    const size_t flags_end = kPeerFlagsOffset + (size_t)batch * kNumQHeads * 4;
    return (flags_end + 255) & ~(size_t)255;
}
__host__ __device__ inline size_t peer_push_offset(int batch) {
    return peer_data_offset(batch) + 2 * (size_t)batch * kNumQHeads * kPartialFloats * sizeof(float);
}
constexpr size_t kPushFlagsBytes = 256;  // kMaxPeers x 8 KV heads x u32
// Push rows of the fused exchange: [2 parities][kMaxPeers source ranks][32 Q heads][130] 64-bit words,
// each (value, epoch): acc[128], m, l.
constexpr int kPushRowWords = kHeadDim + 2;
constexpr size_t kPushRowsBytes = 2 * (size_t)kMaxPeers * kNumQHeads * kPushRowWords * sizeof(uint64_t);
static_assert(kMaxPeers * kNumKVHeads * 4 <= (int)kPushFlagsBytes, "push flags fit");

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Relaxed system-scope store: after one fence.acq_rel.sys it completes a
// release of everything before the fence (fence + relaxed store), without the
// per-store wait of st.release.
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with parity `parity` to complete; false after the timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitTimeoutCycles) return false;
    }
    return true;
}

// L2 policy for streamed-once K/V rows.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Tiled TMA copy of one box of a 3-D tensor map into this CTA's shared memory,
// completing the box's bytes of transaction count on `bar`.  The innermost
// coordinate is always 0 (head_dim starts a row), so it is 16-byte aligned.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// L2 prefetch of one TMA box (no shared memory, no barrier).  A prefetch only
// moves lines into the device-coherent L2: issued before the dependency wait it
// cannot make a later load see stale data.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// L2 prefetch of `bytes` (a multiple of 16) at a 16-byte aligned address.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Bulk (non-tensor) TMA copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  16-byte aligned addresses, size a
// multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also returns whether any participating thread passed true.
__device__ __forceinline__ bool named_barrier_or(int id, int threads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %3, 0;\n\t"
        "barrier.red.or.pred q, %1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(threads), "r"(v ? 1u : 0u)
        : "memory");
    return r != 0;
}

// Arrive on a named barrier without waiting (the producer side of a hand-off:
// shared-memory writes before it are visible to the threads that bar.sync on it).
__device__ __forceinline__ void named_barrier_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Thread-block cluster barrier (release on arrive, acquire on wait) and loads
// from another CTA's shared memory in the cluster.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ float2 ld_cluster_f32x2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(smem_addr(p)));
    return r;
}

__device__ __forceinline__ uint2 lds64(const void* p) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(smem_addr(p)));
    return r;
}

__device__ __forceinline__ float4 lds128f(const void* p) {
    float4 r;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "r"(smem_addr(p)));
    return r;
}

// Two BF16 codes in one 32-bit word -> (element 2j, element 2j+1) as float2.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// 2^x for x <= 0 with one MUFU.EX2 (PTX ex2.approx.ftz: relative error below 2^-22,
// results below 2^-126 flushed to zero, which only drops weights under 2^-126 of the row max).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------------------
// RoPE phase.  Pair i turns by theta^(-2i/128) / (2*pi) turns per position,
// held as an unsigned Q0.64 fraction: the product with a position wraps
// modulo one turn exactly.  This is the numerically-controlled-oscillator idea
// of rope_unit.v:159-172 with a 64-bit phase, followed by sincospif on the
// reduced angle instead of a 14-bit BF16 ROM.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 rope_factor(uint64_t step, int64_t pos) {
    const uint64_t ph = step * static_cast<uint64_t>(pos);
    const float x = __ll2float_rn(static_cast<long long>(ph)) * 0x1p-63f;  // 2*turns in [-1, 1)
    float s, c;
    sincospif(x, &s, &c);
    return make_float2(c, s);
}

}  // namespace gqa
