// gqa_decode.cu -- split-KV flash-decoding kernel for GQA (32 Q heads over 8 KV
// heads, head_dim 128) on sm_100a, plus the cross-shard log-sum-exp combine and
// a stand-alone RoPE kernel.
//
// What one CTA computes: the attention of the 4 Q heads of one KV head h of one
// sequence b over a contiguous range of that sequence's visible keys (a
// "split").  This is the reference's per-KV-head group loop
// (gqa_controller.v:140-277: Q group -> K position -> block) with the key loop
// cut into splits so that every SM streams K/V rows at once.
//
// Pipeline (per CTA):
//   warp 8      producer: bulk-copies 64-key K and V tiles (16 KB each) into a
//               4-stage shared-memory ring, one mbarrier per stage and direction.
//   warps 0..7  consumers: warp c owns keys [8c, 8c+8) of every tile, four at a
//               time: 8 lanes per key, each lane 8 rotate_half pairs (16 of the
//               128 dims).  Per key: RoPE of K (rope_unit.v), the 4 Q.K dot
//               products in FP32 (bf16_dot_product_mac.v + scale_unit.v), a
//               3-level shuffle reduction, the hardware mask (score_tag_fifo /
//               gqa_attention_wrapper.v:279), online softmax in log2 units
//               (flash_softmax.v:233-490) and the P.V accumulation
//               (output_accumulator.v:244-536) with each lane owning 4 dims.
//   epilogue    the 8 warps' (m, l, acc) merge through shared memory; a sequence
//               with one split writes BF16 rows directly (O * 1/l,
//               output_accumulator.v:546-687), otherwise each split publishes
//               an FP32 partial to the workspace and the last split of (b, h)
//               to arrive merges them.
#include "gqa_device.cuh"
#include "gqa_internal.h"

namespace gqa {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kTileKeys = 64;
constexpr int kStages = 4;
constexpr int kKeysPerWarp = kTileKeys / kConsumerWarps;  // 8: two groups of 4
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kTileBytes = kTileKeys * kRowBytes;
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kReanchorTiles = 32;  // exact RoPE phase every 32 tiles (2048 keys)

constexpr int kOffBars = kStages * kStageBytes;
constexpr int kOffP = kOffBars + 2 * kStages * 8;
constexpr int kOffAlpha = kOffP + kConsumerWarps * kKeysPerWarp * kGroup * 4;
constexpr int kOffInfo = kOffAlpha + kConsumerWarps * kGroup * 4;
constexpr int kSmemBytes = kOffInfo + 64;
static_assert(kConsumerWarps * kGroup * kPartialFloats * 4 <= kOffBars, "combine buffer must fit the ring");

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

// Complex multiply of (re, im) pairs held as float2 lanes: (ar + i ai) * (br + i bi).
__device__ __forceinline__ void cmul2(float2 ar, float2 ai, float2 br, float2 bi, float2& cr, float2& ci) {
    const float2 nbi = make_float2(-bi.x, -bi.y);
    cr = __ffma2_rn(ar, br, __fmul2_rn(ai, nbi));
    ci = __ffma2_rn(ar, bi, __fmul2_rn(ai, br));
}

// Exact RoPE factors of this lane's 8 pairs (8g .. 8g+7) at absolute position pos.
__device__ __forceinline__ void rope_factors8(const DecodeArgs& a, int g, int64_t pos, float2 (&wr)[4],
                                              float2 (&wi)[4]) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const float2 f0 = rope_factor(a.rope_step[8 * g + 2 * jj], pos);
        const float2 f1 = rope_factor(a.rope_step[8 * g + 2 * jj + 1], pos);
        wr[jj] = make_float2(f0.x, f1.x);
        wi[jj] = make_float2(f0.y, f1.y);
    }
}

__device__ __forceinline__ void write_result(const DecodeArgs& a, int b, int qh, int dim, float acc, float m,
                                             float l) {
    if (a.flags & 1u) {
        float* o = static_cast<float*>(a.out) + (int64_t)b * a.o_bstride + (int64_t)qh * a.o_hstride;
        o[dim] = acc;
        if (dim == 0) {
            o[128] = m;
            o[129] = l;
            o[130] = 0.f;
            o[131] = 0.f;
        }
    } else {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + (int64_t)b * a.o_bstride + (int64_t)qh * a.o_hstride;
        o[dim] = __float2bfloat16_rn(acc / l);
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* empty = full + kStages;
    float* pbuf = reinterpret_cast<float*>(smem + kOffP);
    float* abuf = reinterpret_cast<float*>(smem + kOffAlpha);
    int* info = reinterpret_cast<int*>(smem + kOffInfo);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.x % kNumKVHeads;
    const int gsplit = blockIdx.x / kNumKVHeads;

    // ---- which (sequence, split) this CTA owns: prefix sum of splits per sequence
    if (warp == 0) {
        int b = 0, split = gsplit;
        if (a.descs != nullptr) {
            int base = 0;
            b = -1;
            for (int b0 = 0; b0 < a.batch && b < 0; b0 += 32) {
                const int bb = b0 + lane;
                const int ns = bb < a.batch ? seq_splits(a.descs[bb], a.chunk) : 0;
                int incl = ns;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                const int excl = incl - ns;
                const bool hit = bb < a.batch && gsplit >= base + excl && gsplit < base + incl;
                const unsigned m = __ballot_sync(0xffffffffu, hit);
                if (m) {
                    const int src = __ffs(m) - 1;
                    b = b0 + src;
                    split = gsplit - base - __shfl_sync(0xffffffffu, excl, src);
                }
                base += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        if (lane == 0) {
            info[0] = b;
            info[1] = split;
        }
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const int b = info[0];
    const int split = info[1];
    if (b < 0) return;  // grid larger than the plan: nothing to do (uniform per CTA)
    const SeqDesc d = a.descs != nullptr ? a.descs[b] : a.single;
    const int n_keys = seq_key_count(d);
    const int n_split = seq_splits(d, a.chunk);
    const int key0 = split * a.chunk;
    const int cnt = max(0, min(a.chunk, n_keys - key0));
    const int n_tiles = (cnt + kTileKeys - 1) / kTileKeys;
    const int64_t first_pos = (int64_t)d.pos_begin + key0;
    const int64_t first_row = d.kv_start + key0;

    // ======================= producer warp =======================
    if (warp == kConsumerWarps) {
        const __nv_bfloat16* kb = a.k + first_row * a.k_pstride + (int64_t)h * a.k_hstride;
        const __nv_bfloat16* vb = a.v + first_row * a.v_pstride + (int64_t)h * a.v_hstride;
        const bool k_rows_contig = a.k_pstride == kHeadDim;
        const bool v_rows_contig = a.v_pstride == kHeadDim;
        const uint64_t pol = l2_evict_first_policy();
        int issued = 0;
        bool ok = true;
        for (int t = 0; t < n_tiles; ++t) {
            const int st = t % kStages;
            if (t >= kStages) ok = mbar_wait(&empty[st], ((t / kStages) - 1) & 1);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            const int rows = min(kTileKeys, cnt - t * kTileKeys);
            uint8_t* kd = smem + st * kStageBytes;
            uint8_t* vd = kd + kTileBytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[st], rows * 2 * kRowBytes);
            __syncwarp();
            const __nv_bfloat16* ks = kb + (int64_t)t * kTileKeys * a.k_pstride;
            const __nv_bfloat16* vs = vb + (int64_t)t * kTileKeys * a.v_pstride;
            if (k_rows_contig) {
                if (lane == 0) bulk_load(kd, ks, rows * kRowBytes, &full[st], pol);
            } else {
                for (int r = lane; r < rows; r += 32)
                    bulk_load(kd + r * kRowBytes, ks + (int64_t)r * a.k_pstride, kRowBytes, &full[st], pol);
            }
            if (v_rows_contig) {
                if (lane == 1) bulk_load(vd, vs, rows * kRowBytes, &full[st], pol);
            } else {
                for (int r = lane; r < rows; r += 32)
                    bulk_load(vd + r * kRowBytes, vs + (int64_t)r * a.v_pstride, kRowBytes, &full[st], pol);
            }
            issued = t + 1;
        }
        if (!ok && lane == 0) atomicOr(a.ws_status, kDevStatusTimeout);
        // Do not leave while copies into this CTA's shared memory are in flight.
        for (int t = max(0, issued - kStages); t < issued; ++t) mbar_wait(&full[t % kStages], (t / kStages) & 1);
        return;
    }

    // ======================= consumer warps =======================
    const int c = warp;
    const int slot = lane >> 3;  // key within the group of 4 this step handles
    const int g = lane & 7;      // pairs 8g .. 8g+7 (dims 8g..8g+7 and 64+8g..64+8g+7)
    const int hh = g >> 1;       // Q head whose score this lane holds after the reduction
    const int qpos = d.query_position;

    if (a.mask_out != nullptr && split == 0 && h == 0) {
        const int n_pad = ((d.seq_len + a.kv_block_len - 1) / a.kv_block_len) * a.kv_block_len;
        for (int p = threadIdx.x; p < n_pad; p += kConsumerThreads)
            a.mask_out[(int64_t)b * a.mask_stride + p] = key_valid(p, d.seq_len, qpos) ? 1 : 0;
    }

    // Q rows of the group, rotated at QUERY_POSITION and pre-scaled by scale*log2(e).
    float2 qr[kGroup][4], qi[kGroup][4];
    {
        float2 wr[4], wi[4];
        rope_factors8(a, g, qpos, wr, wi);
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq) {
            const __nv_bfloat16* qrow = a.q + (int64_t)b * a.q_bstride + (int64_t)(h * kGroup + hq) * a.q_hstride;
            const uint4 xr = *reinterpret_cast<const uint4*>(qrow + 8 * g);
            const uint4 xi = *reinterpret_cast<const uint4*>(qrow + kPairs + 8 * g);
            const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
            const uint32_t yw[4] = {xi.x, xi.y, xi.z, xi.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                float2 re, im;
                cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), wr[jj], wi[jj], re, im);
                qr[hq][jj] = __fmul2_rn(re, f2(a.qscale));
                qi[hq][jj] = __fmul2_rn(im, f2(a.qscale));
            }
        }
    }

    // RoPE factors of this lane's key in step 0 of the current tile, and the
    // fixed rotations that advance them by 4 keys and by one tile.
    float2 wr[4], wi[4], sr[4], si[4], tr[4], ti[4];
    rope_factors8(a, g, first_pos + c * kKeysPerWarp + slot, wr, wi);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const float2 s0 = a.rot_step[8 * g + 2 * jj], s1 = a.rot_step[8 * g + 2 * jj + 1];
        const float2 t0 = a.rot_tile[8 * g + 2 * jj], t1 = a.rot_tile[8 * g + 2 * jj + 1];
        sr[jj] = make_float2(s0.x, s1.x);
        si[jj] = make_float2(s0.y, s1.y);
        tr[jj] = make_float2(t0.x, t1.x);
        ti[jj] = make_float2(t0.y, t1.y);
    }

    float m_run = -INFINITY;  // running max (log2 units) of head hh
    float l_run = 0.f;        // running sum of this lane's key slot for head hh
    float2 acc0[kGroup], acc1[kGroup];  // dims (4*lane, +1) and (4*lane+2, +3) of each head
#pragma unroll
    for (int hq = 0; hq < kGroup; ++hq) acc0[hq] = acc1[hq] = make_float2(0.f, 0.f);
    float* pw = pbuf + c * (kKeysPerWarp * kGroup);

    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
        const int st = t % kStages;
        if (!mbar_wait(&full[st], (t / kStages) & 1)) {
            ok = false;
            break;
        }
        const uint8_t* kt = smem + st * kStageBytes;
        const uint8_t* vt = kt + kTileBytes;
        const int rows = min(kTileKeys, cnt - t * kTileKeys);
        const int64_t tile_pos = first_pos + (int64_t)t * kTileKeys;

        float sc[2];
#pragma unroll
        for (int step = 0; step < 2; ++step) {
            const int r = c * kKeysPerWarp + step * 4 + slot;
            float2 ur[4], ui[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                if (step == 0) {
                    ur[jj] = wr[jj];
                    ui[jj] = wi[jj];
                } else {
                    cmul2(wr[jj], wi[jj], sr[jj], si[jj], ur[jj], ui[jj]);
                }
            }
            const uint4 kre = lds128(kt + r * kRowBytes + g * 16);
            const uint4 kim = lds128(kt + r * kRowBytes + 128 + g * 16);
            const uint32_t xw[4] = {kre.x, kre.y, kre.z, kre.w};
            const uint32_t yw[4] = {kim.x, kim.y, kim.z, kim.w};
            float2 rr[4], ri[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
                cmul2(bf16x2_to_float2(xw[jj]), bf16x2_to_float2(yw[jj]), ur[jj], ui[jj], rr[jj], ri[jj]);
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
            // Sum the 4 head scores over the 8 lanes of this key (lane bits 0..2);
            // lane ends with head hh = (bit2, bit1).
            const bool b2 = lane & 4, b1 = lane & 2;
            const float t0 = (b2 ? s[2] : s[0]) + __shfl_xor_sync(0xffffffffu, b2 ? s[0] : s[2], 4);
            const float t1 = (b2 ? s[3] : s[1]) + __shfl_xor_sync(0xffffffffu, b2 ? s[1] : s[3], 4);
            float u = (b1 ? t1 : t0) + __shfl_xor_sync(0xffffffffu, b1 ? t0 : t1, 2);
            u += __shfl_xor_sync(0xffffffffu, u, 1);
            const bool valid = r < rows && key_valid(tile_pos + r, d.seq_len, qpos);
            sc[step] = valid ? u : -INFINITY;
        }
        // Advance the lane's RoPE factors by one tile (exactly every kReanchorTiles).
        if (((t + 1) % kReanchorTiles) == 0) {
            rope_factors8(a, g, tile_pos + kTileKeys + c * kKeysPerWarp + slot, wr, wi);
        } else {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                float2 nr, ni;
                cmul2(wr[jj], wi[jj], tr[jj], ti[jj], nr, ni);
                wr[jj] = nr;
                wi[jj] = ni;
            }
        }

        // Online softmax for head hh over this warp's 8 keys.
        float mx = fmaxf(sc[0], sc[1]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run, mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = exp2f(m_run - m_use);
        const float p0 = exp2f(sc[0] - m_use);
        const float p1 = exp2f(sc[1] - m_use);
        l_run = l_run * alpha + (p0 + p1);
        m_run = m_new;
        if ((g & 1) == 0) {
            pw[slot * kGroup + hh] = p0;
            pw[(4 + slot) * kGroup + hh] = p1;
            if (slot == 0) abuf[c * kGroup + hh] = alpha;
        }
        __syncwarp();
        const float4 al = lds128f(abuf + c * kGroup);
        const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
        for (int hq = 0; hq < kGroup; ++hq) {
            acc0[hq] = __fmul2_rn(acc0[hq], f2(alv[hq]));
            acc1[hq] = __fmul2_rn(acc1[hq], f2(alv[hq]));
        }
        const int nr = rows - c * kKeysPerWarp;  // keys of this warp present in the tile
#pragma unroll
        for (int rr = 0; rr < kKeysPerWarp; ++rr) {
            if (rr < nr) {
                const float4 pp = lds128f(pw + rr * kGroup);
                const uint2 vv = lds64(vt + (c * kKeysPerWarp + rr) * kRowBytes + lane * 8);
                const float2 v0 = bf16x2_to_float2(vv.x), v1 = bf16x2_to_float2(vv.y);
                const float pv[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
                for (int hq = 0; hq < kGroup; ++hq) {
                    acc0[hq] = __ffma2_rn(f2(pv[hq]), v0, acc0[hq]);
                    acc1[hq] = __ffma2_rn(f2(pv[hq]), v1, acc1[hq]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (!ok && lane == 0) atomicOr(a.ws_status, kDevStatusTimeout);

    l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);

    // ---- merge the 8 warps through shared memory (the ring is free now)
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

    const int tid = threadIdx.x;
    const int dim = tid & 127;
    float res_acc[2], res_m[2], res_l[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int hq = (tid >> 7) + 2 * i;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cb[(w * kGroup + hq) * kPartialFloats + 128]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float* row = cb + (w * kGroup + hq) * kPartialFloats;
            const float f = exp2f(row[128] - Mu);
            L = fmaf(row[129], f, L);
            O = fmaf(row[dim], f, O);
        }
        res_acc[i] = O;
        res_m[i] = M;
        res_l[i] = L;
    }

    if (n_split == 1) {
#pragma unroll
        for (int i = 0; i < 2; ++i) write_result(a, b, h * kGroup + (tid >> 7) + 2 * i, dim, res_acc[i], res_m[i], res_l[i]);
        return;
    }

    // ---- publish this split's partial; the last split of (b, h) merges them
    float* part = a.ws_partials + ((int64_t)gsplit * kNumKVHeads + h) * kGroup * kPartialFloats;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float* row = part + ((tid >> 7) + 2 * i) * kPartialFloats;
        row[dim] = res_acc[i];
        if (dim == 0) {
            row[128] = res_m[i];
            row[129] = res_l[i];
        }
    }
    __threadfence();
    named_barrier_sync(1, kConsumerThreads);
    if (tid == 0) {
        const unsigned old = atomicAdd(&a.ws_counters[b * kNumKVHeads + h], 1u);
        info[2] = old == (unsigned)(n_split - 1) ? 1 : 0;
    }
    named_barrier_sync(1, kConsumerThreads);
    if (info[2] == 0) return;
    __threadfence();
    const int gbase = gsplit - split;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int hq = (tid >> 7) + 2 * i;
        float M = -INFINITY;
        for (int s = 0; s < n_split; ++s) {
            const float* row = a.ws_partials + (((int64_t)(gbase + s) * kNumKVHeads + h) * kGroup + hq) * kPartialFloats;
            M = fmaxf(M, __ldcg(row + 128));
        }
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int s = 0; s < n_split; ++s) {
            const float* row = a.ws_partials + (((int64_t)(gbase + s) * kNumKVHeads + h) * kGroup + hq) * kPartialFloats;
            const float f = exp2f(__ldcg(row + 128) - Mu);
            L = fmaf(__ldcg(row + 129), f, L);
            O = fmaf(__ldcg(row + dim), f, O);
        }
        write_result(a, b, h * kGroup + hq, dim, O, M, L);
    }
    if (tid == 0) a.ws_counters[b * kNumKVHeads + h] = 0u;
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

}  // namespace

int decode_tile_keys() { return kTileKeys; }
size_t decode_smem_bytes() { return kSmemBytes; }

cudaError_t decode_prepare(int device) {
    (void)device;
    return cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream) {
    decode_kernel<<<grid, kThreads, kSmemBytes, stream>>>(a);
    return cudaGetLastError();
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

}  // namespace gqa
