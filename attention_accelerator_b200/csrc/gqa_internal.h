// gqa_internal.h -- host-side launch entry points of the kernels (library-internal).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <initializer_list>

namespace gqa {

// GQA_OK when every non-null pointer is memory the current GPU's kernels and
// TMA units address directly: a device allocation of this GPU or managed
// memory.  Host memory (pageable or pinned) and another GPU's allocations give
// GQA_ERR_MEMORY, before anything is launched, so that a wrong pointer at the C
// boundary becomes a status instead of a memory fault on the GPU.
int check_device_memory(std::initializer_list<const void*> ptrs);

struct DecodeArgs;
struct RopeTable;

// Device address of the RoPE table for `theta` on the current device, built and
// uploaded on first use (a synchronous copy: first use must precede stream
// capture).  At most kRopeTableSlots distinct thetas per device.
constexpr int kRopeTableSlots = 4;
cudaError_t rope_table_for(double theta, const RopeTable** table, bool* out_of_slots);

int decode_tile_keys();
int decode_max_splits();
size_t decode_smem_bytes();
cudaError_t decode_prepare(int device);
// Most splits of one sequence the in-cluster merge takes, and how many clusters
// of `cluster` decode CTAs the current device can hold at once (0: none).
int decode_max_cluster_splits();
// Most splits of one sequence the last-split merge takes (more: split_merge_kernel).
int decode_last_merge_max_splits();
int decode_cluster_capacity(int cluster);
// Decode of a.batch sequences in total_splits splits (grid total_splits x 8 CTAs,
// then split_merge_kernel when a sequence has several splits), or, for
// a.cluster > 0, one sequence in a.cluster splits merged inside the clusters.
cudaError_t launch_decode(const DecodeArgs& a, int total_splits, cudaStream_t stream);
cudaError_t launch_combine(const float* parts, int n_parts, int64_t part_stride, int64_t batch_stride, int batch,
                           void* out, int64_t o_bstride, int64_t o_hstride, cudaStream_t stream);
cudaError_t launch_rope_k_cache(const void* k, void* out, const int32_t* pos, int n_positions, int64_t pos_stride,
                                int64_t head_stride, const uint64_t* step, cudaStream_t stream);
cudaError_t launch_rope_rows(const void* x, const int32_t* pos, float* out, int rows, const uint64_t* step,
                             cudaStream_t stream);

// Chunked multi-query decode (tensor cores): up to 128 consecutive query
// positions per sequence, one CTA per (sequence, Q head).
struct ChunkLaunch {
    CUtensorMap kmap, vmap;  // 4-D K/V maps, 128-byte swizzle, box 64 dims x 64 rows
    int kv_rows_inner;
    const void* q;
    void* out;
    int64_t q_bstride, q_istride, q_hstride;
    int64_t o_bstride, o_istride, o_hstride;
    int batch, seq_len, first_pos, n_queries;
    float qscale;
    uint32_t* status;
    const RopeTable* rope;
    int full_units, split;  // key-range split of the last wave's units (chunked_split_plan)
    float* partials;        // chunked_partial_bytes of workspace for their partial rows
};
void chunked_split_plan(int batch, int seq_len, int first_pos, int n_queries, int sms, int* full_units, int* split);
size_t chunked_partial_bytes(int batch, int full_units, int split);
size_t chunked_smem_bytes();
int chunked_max_queries();
int chunked_tile_keys();
cudaError_t chunked_prepare();
cudaError_t launch_chunked(const ChunkLaunch& l, cudaStream_t stream);

// Long-context exchange of per-GPU partial rows over peer memory + LSE combine.
size_t peer_buffer_bytes(int batch);
cudaError_t launch_combine_peers(const float* local, int64_t part_bstride, const uint64_t* peer_bases, int world,
                                 int rank, int batch, void* out, int64_t o_bstride, int64_t o_hstride,
                                 uint32_t* status, cudaStream_t stream);

}  // namespace gqa
