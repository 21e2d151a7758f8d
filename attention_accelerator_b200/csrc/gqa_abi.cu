// gqa_abi.cu -- the extern "C" boundary declared in include/gqa_b200.h:
// host-side validation (the reference's start-time config_error), planning of
// key splits, workspace layout, argument packing and kernel launches.
#include "gqa_b200.h"
#include "gqa_device.cuh"
#include "gqa_internal.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <queue>
#include <vector>
#include <mutex>

static_assert(sizeof(gqa_seq_desc) == sizeof(gqa::SeqDesc), "descriptor layout");
static_assert(sizeof(gqa_partial_row) == gqa::kPartialFloats * sizeof(float), "partial row layout");

namespace gqa {

int check_device_memory(std::initializer_list<const void*> ptrs) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_CUDA;
    for (const void* ptr : ptrs) {
        if (ptr == nullptr) continue;  // each entry point checks its required pointers itself
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
            (void)cudaGetLastError();  // leave no error behind for the launch checks that follow
            return GQA_ERR_MEMORY;
        }
        if (at.type == cudaMemoryTypeManaged) continue;
        if (at.type != cudaMemoryTypeDevice || at.device != dev) return GQA_ERR_MEMORY;
    }
    return GQA_OK;
}

}  // namespace gqa

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kWsHeaderBytes = 256;  // status word at 0, per-KV-head arrival counters at 64, work queue at 128
constexpr size_t kWsArrivalsOffset = 64;
constexpr size_t kWsWorkOffset = 128;  // a batch's work queue: next item, CTAs done
constexpr int kMinChunk = gqa::kDecodeTileKeys;  // keys: one pipeline tile
constexpr int kMinChunkMultiWave = 256;
constexpr int kMaxWaves = 16;
constexpr int kOverheadKeys = 64;    // per-CTA prologue/epilogue cost, in key-equivalents
constexpr int kBatchOverheadKeys = 128;  // the same for a batch's splits (they also pass through split_merge_kernel)
// What merging a single sequence's splits adds to its latency, in pipeline
// tiles of one CTA: the last split's arrival and L2 round trip, or a cluster
// barrier and distributed-shared-memory round trip.
constexpr double kLastSplitMergeTiles = 1.5;
constexpr double kClusterMergeTiles = 0.3;

struct DeviceInfo {
    bool init = false;
    int status = GQA_OK;
    int sms = 0;
    int cluster_cap[17] = {};  // decode clusters of n CTAs the device holds at once
    bool cluster_asked[17] = {};  // cluster_cap[n] is known
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

// Current device's SM count; prepares the kernels once per device.
int current_device(int* sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GQA_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceInfo& di = g_dev[dev];
    if (!di.init) {
        int major = 0, minor = 0, n = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            return GQA_ERR_CUDA;
        }
        if (major != 10 || minor != 0) {
            di.status = GQA_ERR_UNSUPPORTED_DEVICE;
        } else if (gqa::decode_prepare(dev) != cudaSuccess || gqa::chunked_prepare() != cudaSuccess) {
            di.status = GQA_ERR_CUDA;
        }
        di.sms = n;
        di.init = true;
    }
    if (di.status != GQA_OK) return di.status;
    *sms = di.sms;
    return GQA_OK;
}

// Decode clusters of n CTAs the current device can hold at once (cached).
int cluster_capacity(int n) {
    int dev = 0;
    if (n < 2 || n > 16 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceInfo& di = g_dev[dev];
    if (!di.cluster_asked[n]) {
        di.cluster_cap[n] = gqa::decode_cluster_capacity(n);
        di.cluster_asked[n] = true;
    }
    return di.cluster_cap[n];
}

// cuTensorMapEncodeTiled from the driver, fetched once through the runtime (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D tensor map over K or V: (head_dim, row, head) when rows are the smaller
// stride (head-major), else (head_dim, head, row).  One box = one tile of
// consecutive rows of one head; rows past `rows` read as zeros.  `heads`: the
// KV heads the tensor holds (8, or a head-sharded call's range).
int make_kv_map(CUtensorMap* map, const void* base, int64_t pos_stride, int64_t head_stride, int64_t rows,
                int* rows_inner, int heads = gqa::kNumKVHeads) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return GQA_ERR_CUDA;
    const cuuint64_t tile = (cuuint64_t)gqa::decode_tile_keys();
    cuuint64_t dims[3];
    cuuint64_t strides[2];
    cuuint32_t box[3];
    const cuuint32_t estr[3] = {1, 1, 1};
    if (pos_stride <= head_stride) {
        dims[0] = gqa::kHeadDim; dims[1] = (cuuint64_t)rows; dims[2] = (cuuint64_t)heads;
        strides[0] = (cuuint64_t)pos_stride * 2; strides[1] = (cuuint64_t)head_stride * 2;
        box[0] = gqa::kHeadDim; box[1] = (cuuint32_t)tile; box[2] = 1;
        *rows_inner = 1;
    } else {
        dims[0] = gqa::kHeadDim; dims[1] = (cuuint64_t)heads; dims[2] = (cuuint64_t)rows;
        strides[0] = (cuuint64_t)head_stride * 2; strides[1] = (cuuint64_t)pos_stride * 2;
        box[0] = gqa::kHeadDim; box[1] = 1; box[2] = (cuuint32_t)tile;
        *rows_inner = 0;
    }
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GQA_OK : GQA_ERR_ALIGNMENT;
}

// 4-D tensor map over a batch of K or V caches for the chunked kernel:
// (head_dim, head, row, batch) for position-major rows or (head_dim, row, head,
// batch) for head-major; box = 64 dims x 64 rows of one head, 128-byte swizzle
// (the tensor cores' K-major / MN-major operand layout).  Rows past `rows` read
// as zeros.
int make_kv_map_batched(CUtensorMap* map, const void* base, int64_t pos_stride, int64_t head_stride,
                        int64_t batch_stride, int64_t rows, int64_t batch, int* rows_inner) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return GQA_ERR_CUDA;
    const cuuint32_t tile = (cuuint32_t)gqa::chunked_tile_keys();
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (batch > 1 && batch_stride <= 0) return GQA_ERR_ALIGNMENT;
    const cuuint64_t bstride = (cuuint64_t)(batch_stride > 0 ? batch_stride : rows * (pos_stride > head_stride ? pos_stride : head_stride)) * 2;
    if (pos_stride <= head_stride) {
        dims[0] = gqa::kHeadDim; dims[1] = (cuuint64_t)rows; dims[2] = gqa::kNumKVHeads; dims[3] = (cuuint64_t)batch;
        strides[0] = (cuuint64_t)pos_stride * 2; strides[1] = (cuuint64_t)head_stride * 2; strides[2] = bstride;
        box[0] = 64; box[1] = tile; box[2] = 1; box[3] = 1;
        *rows_inner = 1;
    } else {
        dims[0] = gqa::kHeadDim; dims[1] = gqa::kNumKVHeads; dims[2] = (cuuint64_t)rows; dims[3] = (cuuint64_t)batch;
        strides[0] = (cuuint64_t)head_stride * 2; strides[1] = (cuuint64_t)pos_stride * 2; strides[2] = bstride;
        box[0] = 64; box[1] = 1; box[2] = tile; box[3] = 1;
        *rows_inner = 0;
    }
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GQA_OK : GQA_ERR_ALIGNMENT;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride_ok(int64_t s) { return s >= 0 && (s % 8) == 0; }

int check_geometry(const gqa_params* p) {
    if (p->n_q_heads != (uint32_t)gqa::kNumQHeads || p->n_kv_heads != (uint32_t)gqa::kNumKVHeads ||
        p->head_dim != (uint32_t)gqa::kHeadDim || p->tile_dim != 16u)
        return GQA_ERR_GEOMETRY;
    if (p->kv_block_len == 0) return GQA_ERR_KV_BLOCK_LEN;
    if (!(p->scale != 0.f) || !std::isfinite(p->scale)) return GQA_ERR_SCALE;
    if (p->group_size != p->n_q_heads / p->n_kv_heads) return GQA_ERR_GROUP_SIZE;
    if (!(p->rope_theta > 0.f) || !std::isfinite(p->rope_theta)) return GQA_ERR_ROPE_THETA;
    return GQA_OK;
}

int check_layout(const void* q, const void* k, const void* v, const void* out, const gqa_params* p) {
    if (p->flags & ~(GQA_FLAG_PARTIAL_OUT | GQA_FLAG_K_ROTATED | GQA_FLAG_Q_ROTATED)) return GQA_ERR_FLAGS;
    if (!q || !k || !v || !out) return GQA_ERR_NULL_POINTER;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return GQA_ERR_ALIGNMENT;
    if (!stride_ok(p->q_batch_stride) || !stride_ok(p->q_head_stride) || !stride_ok(p->k_head_stride) ||
        !stride_ok(p->v_head_stride) || !stride_ok(p->k_pos_stride) || !stride_ok(p->v_pos_stride) ||
        p->k_pos_stride == 0 || p->v_pos_stride == 0 || p->k_head_stride == 0 || p->v_head_stride == 0)
        return GQA_ERR_ALIGNMENT;
    if (p->flags & GQA_FLAG_PARTIAL_OUT) {
        if (p->out_head_stride < gqa::kPartialFloats || p->out_head_stride % 4 || p->out_batch_stride < 0 ||
            p->out_batch_stride % 4)
            return GQA_ERR_ALIGNMENT;
    } else if (!stride_ok(p->out_head_stride) || !stride_ok(p->out_batch_stride)) {
        return GQA_ERR_ALIGNMENT;  // BF16 rows are written 4 elements at a time
    }
    return gqa::check_device_memory({q, k, v, out, p->mask_out});
}

int check_desc(const gqa::SeqDesc& d, bool need_keys) {
    if (d.seq_len <= 0) return GQA_ERR_SEQ_LEN;
    if (d.query_position < 0 || d.query_position >= d.seq_len) return GQA_ERR_QUERY_POSITION;
    if (d.kv_start < 0 || d.pos_begin < 0 || d.pos_end < d.pos_begin || d.pos_end > d.seq_len)
        return GQA_ERR_KV_RANGE;
    if (need_keys && gqa::seq_key_count(d) == 0) return GQA_ERR_KV_RANGE;
    return GQA_OK;
}

struct Plan {
    int chunk = 0;
    int total_splits = 0;
    int cluster = 0;      // > 0: single sequence, splits merged inside thread-block clusters
    int64_t kv_rows = 1;  // tensor-map row extent: one past the last stored row any key uses
    size_t off_seqinfo = 0, off_partials = 0, ws_bytes = 0;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Keys per split: one wave of CTAs for a single sequence; for a batch, the
// wave count (1..16) that minimises waves x (chunk + per-CTA overhead).  A
// single sequence (allow_cluster) with several splits is instead cut into n
// <= 16 splits merged inside one cluster per KV head when the device holds all
// 8 such clusters at once and that costs fewer tiles per CTA than the one-wave
// plan with its last-split merge.
Plan make_plan(const gqa::SeqDesc* d, int batch, int sms, bool allow_cluster = false, bool clusters_ok = true,
               int heads = gqa::kNumKVHeads) {
    const int slots = sms / heads > 0 ? sms / heads : 1;
    int64_t total = 0, longest = 0;
    for (int b = 0; b < batch; ++b) {
        total += gqa::seq_key_count(d[b]);
        longest = std::max<int64_t>(longest, gqa::seq_key_count(d[b]));
    }
    // The last split of a sequence stages every split's partial in shared memory;
    // a single sequence stays within the in-kernel last-split merge (a KV-head
    // subset on its own GPU would otherwise be cut into more splits than that).
    const int max_splits = batch == 1 ? gqa::decode_last_merge_max_splits() : gqa::decode_max_splits();
    const int64_t min_chunk = (longest + max_splits - 1) / max_splits;
    auto splits_for = [&](int chunk) {
        int64_t s = 0;
        for (int b = 0; b < batch; ++b) s += gqa::seq_splits(d[b], chunk);
        return s;
    };
    auto round8 = [](int64_t x) { return (int)(((x + 7) / 8) * 8); };
    // A batch runs its full-chunk splits first and the shorter last splits after
    // them (decode_kernel's CTA order).  Its cost: that order scheduled greedily
    // on sms/8 machines (the 8 CTAs of a split, one per KV head, side by side),
    // in key-equivalents with a fixed per-split overhead.
    std::vector<int64_t> rems;
    auto schedule_cost = [&](int c) {
        const int machines = std::max(1, slots);
        int64_t full = 0;
        rems.clear();
        for (int b = 0; b < batch; ++b) {
            const int64_t n = gqa::seq_key_count(d[b]);
            full += n / c;
            if (gqa::seq_splits(d[b], c) > n / c) rems.push_back(n % c);
        }
        const double job = (double)c + kBatchOverheadKeys;
        std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
        for (int m = 0; m < machines; ++m)
            free_at.push((double)(full / machines + (m < full % machines ? 1 : 0)) * job);
        double end = 0;
        for (const int64_t r : rems) {
            const double t = free_at.top() + (double)r + kBatchOverheadKeys;
            free_at.pop();
            free_at.push(t);
            end = std::max(end, t);
        }
        while (!free_at.empty()) {
            end = std::max(end, free_at.top());
            free_at.pop();
        }
        return end;
    };
    int best_chunk = 0;
    double best_cost = 0;
    const int max_w = batch == 1 ? 1 : kMaxWaves;
    for (int w = 1; w <= max_w; ++w) {
        int64_t chunk = (total + (int64_t)slots * w - 1) / ((int64_t)slots * w);
        const int floor_chunk = (batch == 1 || w == 1) ? kMinChunk : kMinChunkMultiWave;
        if (chunk < floor_chunk) chunk = floor_chunk;
        if (chunk < min_chunk) chunk = min_chunk;
        const int c = round8(chunk);
        const int64_t ctas = splits_for(c) * heads;
        const int64_t waves = (ctas + sms - 1) / sms;
        const double cost = batch == 1 ? (double)waves * (double)(c + kOverheadKeys) : schedule_cost(c);
        if (best_chunk == 0 || cost < best_cost) {
            best_chunk = c;
            best_cost = cost;
        }
    }
    Plan pl;
    pl.chunk = best_chunk > 0 ? best_chunk : kMinChunk;
    pl.total_splits = (int)splits_for(pl.chunk);
    if (allow_cluster && batch == 1 && pl.total_splits > 1) {
        const int tile = gqa::decode_tile_keys();
        auto tiles = [&](int64_t c) { return (double)((c + tile - 1) / tile); };
        // One split fewer per KV head when that costs no extra tile: the SMs it
        // frees take the next call's CTAs while this call's last splits merge.
        if (slots > 2) {
            const int c = round8(std::max<int64_t>(std::max<int64_t>(kMinChunk, min_chunk),
                                                   (longest + slots - 2) / (slots - 1)));
            if (tiles(c) == tiles(pl.chunk)) {
                pl.chunk = c;
                pl.total_splits = (int)splits_for(c);
            }
        }
        double best = tiles(pl.chunk) + kLastSplitMergeTiles;
        for (int n = gqa::decode_max_cluster_splits(); n >= 2; --n) {
            const int c = round8(std::max<int64_t>(kMinChunk, (longest + n - 1) / n));
            const int ns = (int)splits_for(c);
            const double cost = tiles(c) + kClusterMergeTiles;
            if (clusters_ok && ns >= 2 && cost < best && cluster_capacity(ns) >= heads) {
                best = cost;
                pl.chunk = c;
                pl.total_splits = ns;
                pl.cluster = ns;
            }
        }
    }
    pl.kv_rows = 1;
    for (int b = 0; b < batch; ++b)
        pl.kv_rows = std::max<int64_t>(pl.kv_rows, d[b].kv_start + gqa::seq_key_count(d[b]));
    pl.off_seqinfo = kWsHeaderBytes;
    pl.off_partials = pl.off_seqinfo + align256((size_t)batch * sizeof(int2));
    const size_t partial_splits = pl.cluster > 0 ? 0 : (size_t)pl.total_splits;  // clusters merge on chip
    pl.ws_bytes = pl.off_partials + partial_splits * gqa::kNumKVHeads * gqa::kGroup *
                                        gqa::kPartialFloats * sizeof(float);
    return pl;
}

void rope_steps(double theta, uint64_t* step, float2* rot_step, float2* rot_tile, int tile_keys) {
    const double two_pi = 2.0 * M_PI;
    for (int i = 0; i < gqa::kPairs; ++i) {
        const double inv = std::pow(theta, -2.0 * i / (double)gqa::kHeadDim);
        const double turns_q64 = inv / two_pi * 18446744073709551616.0;  // < 2^62
        step[i] = (uint64_t)std::llround(turns_q64);
        if (rot_step) rot_step[i] = make_float2((float)std::cos(4.0 * inv), (float)std::sin(4.0 * inv));
        if (rot_tile)
            rot_tile[i] = make_float2((float)std::cos(tile_keys * inv), (float)std::sin(tile_keys * inv));
    }
}

gqa::SeqDesc single_desc(const gqa_params* p) {
    gqa::SeqDesc d;
    d.kv_start = 0;
    d.seq_len = (int32_t)p->seq_len;
    d.query_position = (int32_t)p->query_position;
    d.pos_begin = 0;
    d.pos_end = (int32_t)p->seq_len;
    return d;
}

int fill_args(gqa::DecodeArgs& a, const void* q, const void* k, const void* v, void* out, const gqa_params* p,
              void* ws, const Plan& pl, int batch, int head0 = 0, int heads = gqa::kNumKVHeads) {
    std::memset(&a, 0, sizeof(a));
    if (pl.kv_rows > 0x7FFFFFFF) return GQA_ERR_KV_RANGE;
    int inner_k = 0, inner_v = 0;
    int st = make_kv_map(&a.kmap, k, p->k_pos_stride, p->k_head_stride, pl.kv_rows, &inner_k, heads);
    if (st != GQA_OK) return st;
    st = make_kv_map(&a.vmap, v, p->v_pos_stride, p->v_head_stride, pl.kv_rows, &inner_v, heads);
    if (st != GQA_OK) return st;
    if (inner_k != inner_v) return GQA_ERR_ALIGNMENT;  // K and V must share one layout
    a.kv_rows_inner = inner_k;
    a.q = static_cast<const __nv_bfloat16*>(q);
    a.k = static_cast<const __nv_bfloat16*>(k);
    a.v = static_cast<const __nv_bfloat16*>(v);
    a.out = out;
    a.q_bstride = p->q_batch_stride;
    a.q_hstride = p->q_head_stride;
    a.k_pstride = p->k_pos_stride;
    a.k_hstride = p->k_head_stride;
    a.v_pstride = p->v_pos_stride;
    a.v_hstride = p->v_head_stride;
    a.o_bstride = p->out_batch_stride;
    a.o_hstride = p->out_head_stride;
    a.batch = batch;
    a.chunk = pl.chunk;
    a.qscale = (float)((double)p->scale * 1.4426950408889634);
    a.flags = p->flags;
    uint8_t* w = static_cast<uint8_t*>(ws);
    a.ws_status = reinterpret_cast<uint32_t*>(w);
    a.ws_seqinfo = reinterpret_cast<int2*>(w + pl.off_seqinfo);
    a.ws_partials = reinterpret_cast<float*>(w + pl.off_partials);
    a.mask_out = p->mask_out;
    a.mask_stride = p->mask_stride;
    a.kv_block_len = (int)p->kv_block_len;
    a.head0 = head0;
    a.n_heads = heads;
    bool out_of_slots = false;
    if (gqa::rope_table_for((double)p->rope_theta, &a.rope, &out_of_slots) != cudaSuccess) return GQA_ERR_CUDA;
    if (out_of_slots) return GQA_ERR_ROPE_THETA;
    return GQA_OK;
}

}  // namespace

extern "C" {

const char* gqa_status_string(int status) {
    switch (status) {
        case GQA_OK: return "ok";
        case GQA_ERR_GEOMETRY: return "invalid configuration: N_Q_HEADS/N_KV_HEADS/HEAD_DIM/TILE_DIM must be 32/8/128/16";
        case GQA_ERR_SEQ_LEN: return "invalid configuration: SEQ_LEN must be positive";
        case GQA_ERR_N_KV_TILES: return "invalid configuration: N_KV_TILES must equal ceil(SEQ_LEN / KV_BLOCK_LEN)";
        case GQA_ERR_SCALE: return "invalid configuration: SCALE_FACTOR must be non-zero and finite";
        case GQA_ERR_QUERY_POSITION: return "invalid configuration: QUERY_POSITION must be in [0, SEQ_LEN)";
        case GQA_ERR_KV_BLOCK_LEN: return "invalid configuration: KV_BLOCK_LEN must be positive";
        case GQA_ERR_GROUP_SIZE: return "invalid configuration: GROUP_SIZE must equal N_Q_HEADS / N_KV_HEADS";
        case GQA_ERR_NULL_POINTER: return "null tensor pointer";
        case GQA_ERR_ALIGNMENT: return "tensor pointer not 16-byte aligned or stride not a multiple of 8 elements";
        case GQA_ERR_WORKSPACE: return "workspace missing or too small";
        case GQA_ERR_BATCH: return "invalid batch or sequence descriptor";
        case GQA_ERR_KV_RANGE: return "invalid stored key range";
        case GQA_ERR_CUDA: return "CUDA runtime error";
        case GQA_ERR_DEVICE_TIMEOUT: return "a bounded wait inside a kernel timed out";
        case GQA_ERR_UNSUPPORTED_DEVICE: return "current device is not an sm_100 GPU";
        case GQA_ERR_ROPE_THETA: return "invalid rope_theta, or more than 4 distinct rope_theta values on one device";
        case GQA_ERR_FLAGS: return "gqa_params.flags holds a bit this entry point does not support";
        case GQA_ERR_MEMORY: return "a tensor, table or workspace pointer is not memory of the current GPU";
        case GQA_ERR_KV_HEADS: return "KV-head range is empty or outside [0, 8)";
        default: return "unknown status";
    }
}

int gqa_version(void) { return (0 << 16) | (1 << 8) | 0; }

int gqa_device_supported(int device) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
    return major == 10 && minor == 0;
}

int gqa_validate(const gqa_params* p) {
    if (!p) return GQA_ERR_NULL_POINTER;
    // Same conditions, same order, as config_error (gqa_attention_wrapper.v:230-237),
    // then the generator's QUERY_POSITION range (gen_gqa_wrapper_vectors.py:77-78).
    if (p->n_q_heads != (uint32_t)gqa::kNumQHeads || p->n_kv_heads != (uint32_t)gqa::kNumKVHeads ||
        p->head_dim != (uint32_t)gqa::kHeadDim || p->tile_dim != 16u)
        return GQA_ERR_GEOMETRY;
    if (p->seq_len == 0) return GQA_ERR_SEQ_LEN;
    if (p->kv_block_len == 0) return GQA_ERR_KV_BLOCK_LEN;
    if (p->n_kv_tiles != (p->seq_len + p->kv_block_len - 1) / p->kv_block_len) return GQA_ERR_N_KV_TILES;
    if (p->seq_len > 0x7FFFFFFFu) return GQA_ERR_SEQ_LEN;
    const int g = check_geometry(p);
    if (g != GQA_OK) return g;
    if (p->query_position >= p->seq_len) return GQA_ERR_QUERY_POSITION;
    return GQA_OK;
}

size_t gqa_workspace_bytes(const gqa_params* p, const gqa_seq_desc* descs, int batch) {
    if (!p) return 0;
    int sms = 0;
    if (current_device(&sms) != GQA_OK) return 0;
    if (descs == nullptr) {
        if (batch != 1 || gqa_validate(p) != GQA_OK) return 0;
        const gqa::SeqDesc d = single_desc(p);
        return make_plan(&d, 1, sms, true).ws_bytes;
    }
    if (batch < 1) return 0;
    const gqa::SeqDesc* d = reinterpret_cast<const gqa::SeqDesc*>(descs);
    for (int b = 0; b < batch; ++b)
        if (check_desc(d[b], false) != GQA_OK) return 0;
    if (batch > 1) return make_plan(d, batch, sms).ws_bytes;
    // One sequence: enough for gqa_decode_batched and for gqa_decode_exchange (no clusters).
    return std::max(make_plan(d, 1, sms, true).ws_bytes, make_plan(d, 1, sms, true, false).ws_bytes);
}

int gqa_decode_plan(const gqa_params* p, const gqa_seq_desc* descs, int batch, int* splits, int* keys_per_split,
                    int* cluster) {
    if (!p || !splits || !keys_per_split || !cluster) return GQA_ERR_NULL_POINTER;
    int sms = 0;
    int st = current_device(&sms);
    if (st != GQA_OK) return st;
    Plan pl;
    if (descs == nullptr) {
        if (batch != 1) return GQA_ERR_BATCH;
        st = gqa_validate(p);
        if (st != GQA_OK) return st;
        const gqa::SeqDesc d = single_desc(p);
        pl = make_plan(&d, 1, sms, true);
    } else {
        if (batch < 1) return GQA_ERR_BATCH;
        const gqa::SeqDesc* d = reinterpret_cast<const gqa::SeqDesc*>(descs);
        for (int b = 0; b < batch; ++b) {
            st = check_desc(d[b], false);
            if (st != GQA_OK) return st;
        }
        pl = make_plan(d, batch, sms, batch == 1);
    }
    *splits = pl.total_splits;
    *keys_per_split = pl.chunk;
    *cluster = pl.cluster;
    return GQA_OK;
}

int gqa_decode_plan_host(const gqa_params* p, const gqa_seq_desc* descs, int batch, int sms, int* splits,
                         int* keys_per_split) {
    if (!p || !splits || !keys_per_split) return GQA_ERR_NULL_POINTER;
    if (sms < 1) return GQA_ERR_BATCH;
    int st = GQA_OK;
    Plan pl;
    // The planner asks the device only for cluster capacities; with clusters
    // left out (clusters_ok = false) it makes no CUDA call.
    if (descs == nullptr) {
        if (batch != 1) return GQA_ERR_BATCH;
        st = gqa_validate(p);
        if (st != GQA_OK) return st;
        const gqa::SeqDesc d = single_desc(p);
        pl = make_plan(&d, 1, sms, true, false);
    } else {
        if (batch < 1) return GQA_ERR_BATCH;
        const gqa::SeqDesc* d = reinterpret_cast<const gqa::SeqDesc*>(descs);
        for (int b = 0; b < batch; ++b) {
            st = check_desc(d[b], false);
            if (st != GQA_OK) return st;
        }
        pl = make_plan(d, batch, sms, batch == 1, false);
    }
    *splits = pl.total_splits;
    *keys_per_split = pl.chunk;
    return GQA_OK;
}

int gqa_decode(const void* q, const void* k, const void* v, void* out, const gqa_params* p, void* workspace,
               size_t workspace_bytes, void* stream) {
    int st = gqa_validate(p);
    if (st != GQA_OK) return st;
    st = check_layout(q, k, v, out, p);
    if (st != GQA_OK) return st;
    int sms = 0;
    st = current_device(&sms);
    if (st != GQA_OK) return st;
    const gqa::SeqDesc d = single_desc(p);
    const Plan pl = make_plan(&d, 1, sms, true);
    if (!workspace || !aligned16(workspace) || workspace_bytes < pl.ws_bytes) return GQA_ERR_WORKSPACE;
    st = gqa::check_device_memory({workspace});
    if (st != GQA_OK) return st;
    gqa::DecodeArgs a;
    st = fill_args(a, q, k, v, out, p, workspace, pl, 1);
    if (st != GQA_OK) return st;
    a.descs = nullptr;
    a.single = d;
    a.cluster = pl.cluster;
    if (pl.cluster == 0 && pl.total_splits > 1 && pl.total_splits <= gqa::decode_last_merge_max_splits())
        a.ws_arrivals = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsArrivalsOffset);
    if (gqa::launch_decode(a, pl.total_splits, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

size_t gqa_workspace_bytes_heads(const gqa_params* p, int kv_head_count) {
    if (!p || gqa_validate(p) != GQA_OK) return 0;
    if (kv_head_count < 1 || kv_head_count > gqa::kNumKVHeads) return 0;
    int sms = 0;
    if (current_device(&sms) != GQA_OK) return 0;
    const gqa::SeqDesc d = single_desc(p);
    return std::max(make_plan(&d, 1, sms, true, true, kv_head_count).ws_bytes,
                    make_plan(&d, 1, sms, true, false, kv_head_count).ws_bytes);
}

int gqa_decode_heads(const void* q, const void* k, const void* v, void* out, const gqa_params* p,
                     int kv_head_begin, int kv_head_count, void* workspace, size_t workspace_bytes, void* stream) {
    int st = gqa_validate(p);
    if (st != GQA_OK) return st;
    if (kv_head_count < 1 || kv_head_begin < 0 || kv_head_begin + kv_head_count > gqa::kNumKVHeads)
        return GQA_ERR_KV_HEADS;
    st = check_layout(q, k, v, out, p);
    if (st != GQA_OK) return st;
    int sms = 0;
    st = current_device(&sms);
    if (st != GQA_OK) return st;
    const gqa::SeqDesc d = single_desc(p);
    const Plan pl = make_plan(&d, 1, sms, true, true, kv_head_count);
    if (!workspace || !aligned16(workspace) || workspace_bytes < pl.ws_bytes) return GQA_ERR_WORKSPACE;
    st = gqa::check_device_memory({workspace});
    if (st != GQA_OK) return st;
    gqa::DecodeArgs a;
    st = fill_args(a, q, k, v, out, p, workspace, pl, 1, kv_head_begin, kv_head_count);
    if (st != GQA_OK) return st;
    a.descs = nullptr;
    a.single = d;
    a.cluster = pl.cluster;
    if (pl.cluster == 0 && pl.total_splits > 1 && pl.total_splits <= gqa::decode_last_merge_max_splits())
        a.ws_arrivals = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsArrivalsOffset);
    if (gqa::launch_decode(a, pl.total_splits, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_decode_batched(const void* q, const void* k, const void* v, void* out, const gqa_params* p,
                       const gqa_seq_desc* host_descs, const gqa_seq_desc* dev_descs, int batch, void* workspace,
                       size_t workspace_bytes, void* stream) {
    if (!p) return GQA_ERR_NULL_POINTER;
    int st = check_geometry(p);
    if (st != GQA_OK) return st;
    if (batch < 1) return GQA_ERR_BATCH;
    if (!host_descs || !dev_descs) return GQA_ERR_NULL_POINTER;
    st = check_layout(q, k, v, out, p);
    if (st != GQA_OK) return st;
    const gqa::SeqDesc* d = reinterpret_cast<const gqa::SeqDesc*>(host_descs);
    const bool need_keys = (p->flags & GQA_FLAG_PARTIAL_OUT) == 0;
    for (int b = 0; b < batch; ++b) {
        st = check_desc(d[b], need_keys);
        if (st != GQA_OK) return st;
    }
    int sms = 0;
    st = current_device(&sms);
    if (st != GQA_OK) return st;
    // One sequence (e.g. this GPU's shard of a long context) takes the single-
    // sequence plan: splits merged in-kernel, no split-merge launch.
    const Plan pl = make_plan(d, batch, sms, batch == 1);
    if (!workspace || !aligned16(workspace) || workspace_bytes < pl.ws_bytes) return GQA_ERR_WORKSPACE;
    st = gqa::check_device_memory({workspace, dev_descs});
    if (st != GQA_OK) return st;
    gqa::DecodeArgs a;
    st = fill_args(a, q, k, v, out, p, workspace, pl, batch);
    if (st != GQA_OK) return st;
    a.descs = batch == 1 ? nullptr : reinterpret_cast<const gqa::SeqDesc*>(dev_descs);
    a.single = d[0];
    if (batch > 1) {  // decode_queue_kernel: one CTA per SM works through the (split, KV head) items
        a.ws_work = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsWorkOffset);
        a.n_items = pl.total_splits * a.n_heads;
    }
    if (batch == 1) {
        a.cluster = pl.cluster;
        if (pl.cluster == 0 && pl.total_splits > 1 && pl.total_splits <= gqa::decode_last_merge_max_splits())
            a.ws_arrivals = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsArrivalsOffset);
    }
    if (gqa::launch_decode(a, pl.total_splits, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_decode_exchange(const void* q, const void* k, const void* v, void* out, const gqa_params* p,
                        const gqa_seq_desc* shard, const void* const* peer_buffers, int world, int rank, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (!p || !shard || !peer_buffers) return GQA_ERR_NULL_POINTER;
    if (world < 2 || world > gqa::kMaxPeers || rank < 0 || rank >= world) return GQA_ERR_BATCH;
    int st = check_geometry(p);
    if (st != GQA_OK) return st;
    if (p->flags & ~(GQA_FLAG_K_ROTATED | GQA_FLAG_Q_ROTATED)) return GQA_ERR_BATCH;  // final BF16 rows only
    st = check_layout(q, k, v, out, p);
    if (st != GQA_OK) return st;
    const gqa::SeqDesc d = *reinterpret_cast<const gqa::SeqDesc*>(shard);
    st = check_desc(d, false);
    if (st != GQA_OK) return st;
    int sms = 0;
    st = current_device(&sms);
    if (st != GQA_OK) return st;
    const Plan pl = make_plan(&d, 1, sms, true, false);  // single-sequence plan, no clusters
    if (!workspace || !aligned16(workspace) || workspace_bytes < pl.ws_bytes) return GQA_ERR_WORKSPACE;
    st = gqa::check_device_memory({workspace, peer_buffers});  // the array of bases; peers are not local memory
    if (st != GQA_OK) return st;
    gqa::DecodeArgs a;
    st = fill_args(a, q, k, v, out, p, workspace, pl, 1);
    if (st != GQA_OK) return st;
    a.descs = nullptr;
    a.single = d;
    if (pl.total_splits > 1) {
        if (pl.total_splits > gqa::decode_last_merge_max_splits()) return GQA_ERR_KV_RANGE;
        a.ws_arrivals = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsArrivalsOffset);
    }
    a.peer_bases = reinterpret_cast<const uint64_t*>(peer_buffers);
    a.world = world;
    a.rank = rank;
    if (gqa::launch_decode(a, pl.total_splits, static_cast<cudaStream_t>(stream)) != cudaSuccess) return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_combine_partials(const float* partials, int n_parts, int64_t part_stride, int64_t batch_stride, int batch,
                         void* out, int64_t out_batch_stride, int64_t out_head_stride, void* stream) {
    if (!partials || !out) return GQA_ERR_NULL_POINTER;
    if (n_parts < 1 || batch < 1) return GQA_ERR_BATCH;
    if (part_stride < 0 || batch_stride < 0 || out_batch_stride < 0 || out_head_stride < 0) return GQA_ERR_ALIGNMENT;
    int sms = 0;
    int st = current_device(&sms);
    if (st != GQA_OK) return st;
    st = gqa::check_device_memory({partials, out});
    if (st != GQA_OK) return st;
    if (gqa::launch_combine(partials, n_parts, part_stride, batch_stride, batch, out, out_batch_stride,
                            out_head_stride, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_decode_chunked(const void* q, const void* k, const void* v, void* out, const gqa_params* p,
                       const gqa_chunk_params* c, void* workspace, size_t workspace_bytes, void* stream) {
    if (!p || !c) return GQA_ERR_NULL_POINTER;
    if (c->batch < 1 || c->batch > 65535u || c->n_queries < 1 || c->n_queries > (uint32_t)gqa::chunked_max_queries() ||
        c->reserved != 0)
        return GQA_ERR_BATCH;
    if ((uint64_t)c->first_position + c->n_queries > p->seq_len) return GQA_ERR_QUERY_POSITION;
    gqa_params last = *p;
    last.query_position = c->first_position + c->n_queries - 1;
    int st = gqa_validate(&last);
    if (st != GQA_OK) return st;
    if (p->flags != 0 || p->mask_out != nullptr) return GQA_ERR_BATCH;
    st = check_layout(q, k, v, out, p);
    if (st != GQA_OK) return st;
    if (!stride_ok(c->q_query_stride) || !stride_ok(c->out_query_stride) || !stride_ok(c->k_batch_stride) ||
        !stride_ok(c->v_batch_stride))
        return GQA_ERR_ALIGNMENT;
    if (!workspace || !aligned16(workspace) || workspace_bytes < GQA_CHUNKED_WORKSPACE_BYTES) return GQA_ERR_WORKSPACE;
    st = gqa::check_device_memory({workspace});
    if (st != GQA_OK) return st;
    int sms = 0;
    st = current_device(&sms);
    if (st != GQA_OK) return st;
    gqa::ChunkLaunch l;
    std::memset(&l, 0, sizeof(l));
    int inner_k = 0, inner_v = 0;
    st = make_kv_map_batched(&l.kmap, k, p->k_pos_stride, p->k_head_stride, c->k_batch_stride, p->seq_len, c->batch,
                             &inner_k);
    if (st != GQA_OK) return st;
    st = make_kv_map_batched(&l.vmap, v, p->v_pos_stride, p->v_head_stride, c->v_batch_stride, p->seq_len, c->batch,
                             &inner_v);
    if (st != GQA_OK) return st;
    if (inner_k != inner_v) return GQA_ERR_ALIGNMENT;
    l.kv_rows_inner = inner_k;
    l.q = q;
    l.out = out;
    l.q_bstride = p->q_batch_stride;
    l.q_istride = c->q_query_stride;
    l.q_hstride = p->q_head_stride;
    l.o_bstride = p->out_batch_stride;
    l.o_istride = c->out_query_stride;
    l.o_hstride = p->out_head_stride;
    l.batch = (int)c->batch;
    l.seq_len = (int)p->seq_len;
    l.first_pos = (int)c->first_position;
    l.n_queries = (int)c->n_queries;
    l.qscale = (float)((double)p->scale * 1.4426950408889634);
    l.status = static_cast<uint32_t*>(workspace);
    // Split the last wave's units along the keys when the workspace holds their partials.
    gqa::chunked_split_plan((int)c->batch, (int)p->seq_len, (int)c->first_position, (int)c->n_queries, sms,
                            &l.full_units, &l.split);
    const size_t part_bytes = gqa::chunked_partial_bytes((int)c->batch, l.full_units, l.split);
    if (part_bytes == 0 || workspace_bytes < GQA_CHUNKED_WORKSPACE_BYTES + part_bytes) {
        l.full_units = (int)c->batch * gqa::kNumQHeads;
        l.split = 1;
    } else {
        l.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + GQA_CHUNKED_WORKSPACE_BYTES);
    }
    bool out_of_slots = false;
    if (gqa::rope_table_for((double)p->rope_theta, &l.rope, &out_of_slots) != cudaSuccess) return GQA_ERR_CUDA;
    if (out_of_slots) return GQA_ERR_ROPE_THETA;
    if (gqa::launch_chunked(l, static_cast<cudaStream_t>(stream)) != cudaSuccess) return GQA_ERR_CUDA;
    return GQA_OK;
}

size_t gqa_chunked_workspace_bytes(const gqa_params* p, const gqa_chunk_params* c) {
    if (!p || !c || c->batch < 1 || c->batch > 65535u || c->n_queries < 1) return 0;
    int sms = 0;
    if (current_device(&sms) != GQA_OK) return 0;
    int full = 0, split = 1;
    gqa::chunked_split_plan((int)c->batch, (int)p->seq_len, (int)c->first_position, (int)c->n_queries, sms, &full,
                            &split);
    return GQA_CHUNKED_WORKSPACE_BYTES + gqa::chunked_partial_bytes((int)c->batch, full, split);
}

int gqa_rope_rows(const void* x, const int32_t* positions, float* out, int rows, float rope_theta, void* stream) {
    if (!x || !positions || !out) return GQA_ERR_NULL_POINTER;
    if (rows < 0) return GQA_ERR_BATCH;
    if (!(rope_theta > 0.f) || !std::isfinite(rope_theta)) return GQA_ERR_ROPE_THETA;
    if (rows == 0) return GQA_OK;
    int sms = 0;
    int st = current_device(&sms);
    if (st != GQA_OK) return st;
    st = gqa::check_device_memory({x, positions, out});
    if (st != GQA_OK) return st;
    uint64_t step[gqa::kPairs];
    rope_steps((double)rope_theta, step, nullptr, nullptr, 0);
    if (gqa::launch_rope_rows(x, positions, out, rows, step, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_rope_k_cache(const void* k, void* k_rot, const int32_t* positions, int n_positions, int64_t pos_stride,
                     int64_t head_stride, float rope_theta, void* stream) {
    if (!k || !k_rot || !positions) return GQA_ERR_NULL_POINTER;
    if (n_positions < 0) return GQA_ERR_BATCH;
    if (!aligned16(k) || !aligned16(k_rot) || !stride_ok(pos_stride) || !stride_ok(head_stride) || pos_stride == 0 ||
        head_stride == 0)
        return GQA_ERR_ALIGNMENT;
    if (!(rope_theta > 0.f) || !std::isfinite(rope_theta)) return GQA_ERR_ROPE_THETA;
    if (n_positions == 0) return GQA_OK;
    int sms = 0;
    int st = current_device(&sms);
    if (st != GQA_OK) return st;
    st = gqa::check_device_memory({k, k_rot, positions});
    if (st != GQA_OK) return st;
    uint64_t step[gqa::kPairs];
    rope_steps((double)rope_theta, step, nullptr, nullptr, 0);
    if (gqa::launch_rope_k_cache(k, k_rot, positions, n_positions, pos_stride, head_stride, step,
                                 static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

int gqa_rope_phase_rom(uint32_t* phase, int head_dim, double rope_theta) {
    if (!phase) return GQA_ERR_NULL_POINTER;
    if (head_dim <= 0 || head_dim % 2) return GQA_ERR_GEOMETRY;
    if (!(rope_theta > 0.0) || !std::isfinite(rope_theta)) return GQA_ERR_ROPE_THETA;
    const int pairs = head_dim / 2;
    for (int i = 0; i < pairs; ++i) {
        // tools/gen_rope_rom.py:45-47: round(inv_freq * 2**32 / (2*pi)) mod 2**32,
        // Python's round() being round-half-even like nearbyint().
        const double inv = std::pow(rope_theta, -(double)i / pairs);
        const double v = std::nearbyint(inv * 4294967296.0 / (2.0 * M_PI));
        phase[i] = (uint32_t)((uint64_t)v & 0xFFFFFFFFull);
    }
    return GQA_OK;
}

static uint32_t f32_to_bf16_bits(double x) {
    const float f = (float)x;
    uint32_t bits;
    std::memcpy(&bits, &f, 4);
    const uint32_t lsb = (bits >> 16) & 1u;
    return (uint32_t)((((uint64_t)bits + 0x7FFFu + lsb) >> 16) & 0xFFFFu);
}

int gqa_rope_sincos_rom(uint32_t* sincos, int addr_bits) {
    if (!sincos) return GQA_ERR_NULL_POINTER;
    if (addr_bits < 1 || addr_bits > 24) return GQA_ERR_GEOMETRY;
    const int n = 1 << addr_bits;
    for (int i = 0; i < n; ++i) {
        // tools/gen_rope_rom.py:49-54: angle = 2*pi*i/N, {bf16(cos), bf16(sin)}.
        const double a = 2.0 * M_PI * (double)i / (double)n;
        sincos[i] = (f32_to_bf16_bits(std::cos(a)) << 16) | f32_to_bf16_bits(std::sin(a));
    }
    return GQA_OK;
}

int gqa_read_status(void* workspace, void* stream, int* device_status) {
    if (!workspace || !device_status) return GQA_ERR_NULL_POINTER;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t v = 0;
    if (cudaStreamSynchronize(s) != cudaSuccess) return GQA_ERR_CUDA;
    if (cudaMemcpy(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return GQA_ERR_CUDA;
    // After a timed-out wait the arrival counters may be left part-way: clear the header.
    if (v != 0 && cudaMemset(workspace, 0, kWsHeaderBytes) != cudaSuccess) return GQA_ERR_CUDA;
    *device_status = v ? GQA_ERR_DEVICE_TIMEOUT : GQA_OK;
    return GQA_OK;
}

}  // extern "C"
