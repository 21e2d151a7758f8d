// gqa_peer.cu -- the long-context split's exchange of per-GPU partials over
// NVLink peer memory, fused with the log-sum-exp combine.
//
// Every rank owns one exchange buffer (cudaMalloc, shared with the other ranks
// of the node through CUDA IPC handles):
//   [0]   u32 epoch     last completed exchange of this rank
//   [4]   u32 arrivals  CTAs of the running exchange that finished
//   [64]  u32 flag[batch * 32]       epoch whose row (sequence b, Q head h) is published
//   [data] float rows[2][batch * 32][132]   partial rows, double-buffered by epoch parity
// combine_peers_kernel, one CTA per (sequence, Q head) on every rank:
//   1. copy this rank's partial row into rows[e & 1] of its own buffer, then
//      publish flag = e with a system-scope release;
//   2. wait (bounded) until every peer's flag for the row is at least e, with
//      system-scope acquire loads over NVLink;
//   3. read every rank's row and merge:  M = max m_r, O = sum 2^(m_r - M) acc_r,
//      L = sum 2^(m_r - M) l_r, out = BF16(O / L)
//      (flash_softmax.v:233-512 / output_accumulator.v:398-687 applied across GPUs);
//   4. the last CTA to finish advances the epoch.
// Reusing rows[e & 1] at epoch e + 2 is safe: this rank's exchange e + 1 saw
// every peer publish e + 1, which each peer does only after its exchange e, and
// with it every read of this rank's epoch-e rows, has completed (stream order).
// The epoch lives in device memory, so a captured CUDA graph replays correctly.
#include "gqa_b200.h"
#include "gqa_device.cuh"
#include "gqa_internal.h"

#include <cstring>

namespace gqa {

namespace {

constexpr int kHdrFlags = kPeerFlagsOffset;  // byte offset of the flag array

struct PeerArgs {
    const float* local;         // this rank's partial rows [batch][32] with stride part_bstride / 132
    int64_t part_bstride;
    const uint64_t* peer_bases;  // device array: exchange buffer of every rank (own one included)
    int world, rank, batch;
    __nv_bfloat16* out;
    int64_t o_bstride, o_hstride;
    uint32_t* status;
};

__global__ void __launch_bounds__(kHeadDim) combine_peers_kernel(const __grid_constant__ PeerArgs a) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_ok;
    const int row = blockIdx.x;  // b * 32 + qh
    const int b = row / kNumQHeads, qh = row % kNumQHeads;
    const int dim = threadIdx.x;
    uint8_t* mine = reinterpret_cast<uint8_t*>(a.peer_bases[a.rank]);
    uint32_t* hdr = reinterpret_cast<uint32_t*>(mine);
    const size_t data = peer_data_offset(a.batch);
    const size_t rows_per_parity = (size_t)a.batch * kNumQHeads;

    if (dim == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(hdr) + 1u;
    __syncthreads();
    const uint32_t e = s_epoch;
    const size_t slot = ((size_t)(e & 1u) * rows_per_parity + row) * kPartialFloats;

    // 1. publish this rank's row
    const float* src = a.local + (int64_t)b * a.part_bstride + (int64_t)qh * kPartialFloats;
    float* dst = reinterpret_cast<float*>(mine + data) + slot;
    dst[dim] = src[dim];
    if (dim < kPartialFloats - kHeadDim) dst[kHeadDim + dim] = src[kHeadDim + dim];
    __syncthreads();
    if (dim == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        st_release_sys(hdr + kHdrFlags / 4 + row, e);
    }

    // 2. wait for every peer's row of this epoch (bounded)
    if (dim == 0) {
        int ok = 1;
        for (int p = 0; p < a.world && ok; ++p) {
            if (p == a.rank) continue;
            const uint32_t* flag = reinterpret_cast<const uint32_t*>(a.peer_bases[p]) + kHdrFlags / 4 + row;
            if ((int)(ld_acquire_sys(flag) - e) >= 0) continue;
            const long long t0 = clock64();
            while ((int)(ld_acquire_sys(flag) - e) < 0) {
                if (clock64() - t0 > kWaitTimeoutCycles) {
                    ok = 0;
                    break;
                }
            }
        }
        s_ok = ok;
        if (!ok && a.status) atomicOr(a.status, kDevStatusTimeout);
    }
    __syncthreads();

    // 3. merge (volatile loads: another GPU wrote these lines)
    if (s_ok) {
        float M = -INFINITY;
        for (int p = 0; p < a.world; ++p) {
            const volatile float* r =
                reinterpret_cast<const volatile float*>(reinterpret_cast<const uint8_t*>(a.peer_bases[p]) + data) + slot;
            M = fmaxf(M, r[kHeadDim]);
        }
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int p = 0; p < a.world; ++p) {
            const volatile float* r =
                reinterpret_cast<const volatile float*>(reinterpret_cast<const uint8_t*>(a.peer_bases[p]) + data) + slot;
            const float f = exp2f(r[kHeadDim] - Mu);
            L = fmaf(r[kHeadDim + 1], f, L);
            O = fmaf(r[dim], f, O);
        }
        a.out[(int64_t)b * a.o_bstride + (int64_t)qh * a.o_hstride + dim] = __float2bfloat16_rn(O / L);
    }

    // 4. the last CTA advances the epoch
    __syncthreads();
    if (dim == 0) {
        __threadfence();
        const uint32_t done = atomicAdd(hdr + 1, 1u);
        if (done == gridDim.x - 1) {
            hdr[1] = 0u;
            *reinterpret_cast<volatile uint32_t*>(hdr) = e;
        }
    }
}

}  // namespace

size_t peer_buffer_bytes(int batch) { return peer_push_offset(batch) + kPushFlagsBytes + kPushRowsBytes; }

cudaError_t launch_combine_peers(const float* local, int64_t part_bstride, const uint64_t* peer_bases, int world,
                                 int rank, int batch, void* out, int64_t o_bstride, int64_t o_hstride,
                                 uint32_t* status, cudaStream_t stream) {
    PeerArgs a;
    a.local = local;
    a.part_bstride = part_bstride;
    a.peer_bases = peer_bases;
    a.world = world;
    a.rank = rank;
    a.batch = batch;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.o_bstride = o_bstride;
    a.o_hstride = o_hstride;
    a.status = status;
    combine_peers_kernel<<<batch * kNumQHeads, kHeadDim, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace gqa

extern "C" {

size_t gqa_peer_buffer_bytes(int batch) {
    if (batch < 1) return 0;
    return gqa::peer_buffer_bytes(batch);
}

int gqa_peer_buffer_create(size_t bytes, void** buffer, void* ipc_handle) {
    if (!buffer || !ipc_handle) return GQA_ERR_NULL_POINTER;
    if (bytes < 256) return GQA_ERR_WORKSPACE;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return GQA_ERR_CUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return GQA_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return GQA_ERR_CUDA;
    }
    static_assert(sizeof(h) == GQA_PEER_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof(h));
    *buffer = p;
    return GQA_OK;
}

int gqa_peer_buffer_open(const void* ipc_handle, void** buffer) {
    if (!buffer || !ipc_handle) return GQA_ERR_NULL_POINTER;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return GQA_ERR_CUDA;
    *buffer = p;
    return GQA_OK;
}

int gqa_peer_buffer_close(void* buffer) {
    if (!buffer) return GQA_ERR_NULL_POINTER;
    return cudaIpcCloseMemHandle(buffer) == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

int gqa_peer_buffer_destroy(void* buffer) {
    if (!buffer) return GQA_ERR_NULL_POINTER;
    return cudaFree(buffer) == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

int gqa_combine_peers(const float* partials, int64_t partial_batch_stride, const void* const* peer_buffers, int world,
                      int rank, int batch, void* out, int64_t out_batch_stride, int64_t out_head_stride,
                      void* workspace, void* stream) {
    if (!partials || !peer_buffers || !out || !workspace) return GQA_ERR_NULL_POINTER;
    // Every CTA of the exchange must be resident at once (a CTA waits for rows that the
    // peers' CTAs of the same index publish): at most 64 sequences = 2048 small CTAs.
    if (world < 1 || rank < 0 || rank >= world || batch < 1 || batch > 64) return GQA_ERR_BATCH;
    if (partial_batch_stride < (int64_t)gqa::kNumQHeads * gqa::kPartialFloats || out_batch_stride < 0 ||
        out_head_stride < 0)
        return GQA_ERR_ALIGNMENT;
    const int st = gqa::check_device_memory({partials, peer_buffers, out, workspace});  // peer_buffers: the array
    if (st != GQA_OK) return st;
    if (gqa::launch_combine_peers(partials, partial_batch_stride, reinterpret_cast<const uint64_t*>(peer_buffers), world,
                                  rank, batch, out, out_batch_stride, out_head_stride,
                                  static_cast<uint32_t*>(workspace), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return GQA_ERR_CUDA;
    return GQA_OK;
}

}  // extern "C"
