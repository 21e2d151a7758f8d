// gqa_internal.h -- host-side launch entry points of the kernels (library-internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gqa {

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
cudaError_t launch_decode(const DecodeArgs& a, int grid, int total_splits, cudaStream_t stream);
cudaError_t launch_combine(const float* parts, int n_parts, int64_t part_stride, int64_t batch_stride, int batch,
                           void* out, int64_t o_bstride, int64_t o_hstride, cudaStream_t stream);
cudaError_t launch_rope_rows(const void* x, const int32_t* pos, float* out, int rows, const uint64_t* step,
                             cudaStream_t stream);

}  // namespace gqa
