/*
 * gqa_b200.h -- C ABI of the B200 (sm_100a) GQA decode-attention library.
 *
 * The library computes, for one decode token per sequence, the grouped-query
 * attention the reference accelerator implements: RoPE (theta 500000,
 * rotate_half pairing) on Q at QUERY_POSITION and on every K row at its own
 * position, Q.K scaled by `scale`, the hardware mask
 *     key_valid(p) = (p < SEQ_LEN) && (p <= QUERY_POSITION),
 * online softmax, weighted-V accumulation and reciprocal normalisation, for 32
 * Q heads over 8 KV heads (group 4, head_dim 128), producing BF16 [32][128]
 * output rows.
 *
 * Everything here is plain C: pointers, sizes and a `void*` CUDA stream handle
 * (a cudaStream_t; NULL is the legacy default stream).  BF16 tensors are passed
 * as `const void*` to 2-byte BF16 codes.  All device pointers must be 16-byte
 * aligned and every stride (in elements) a multiple of 8.  Tensor, table,
 * descriptor and workspace pointers must be memory of the current GPU (a
 * device allocation or managed memory); host memory, pinned or not, and
 * another GPU's allocations are refused with GQA_ERR_MEMORY before anything is
 * launched.  (The NVLink exchange's peer buffers are the exception: they are
 * reached through a device array of their addresses.)  Calls are
 * asynchronous on `stream` and re-entrant across streams as long as each
 * concurrent call has its own workspace.
 *
 * Status codes: every entry point returns GQA_OK (0) or a positive GQA_ERR_*
 * code.  Configuration errors are detected on the host before anything is
 * launched, mirroring the reference's start-time `config_error`
 * (gqa_attention_wrapper.v:230-237) and the generator's argument checks
 * (pyfiles/gen_gqa_wrapper_vectors.py:57-78).
 */
#ifndef GQA_B200_H
#define GQA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum gqa_status {
    GQA_OK = 0,
    GQA_ERR_GEOMETRY = 1,          /* N_Q_HEADS/N_KV_HEADS/HEAD_DIM/TILE_DIM != 32/8/128/16 */
    GQA_ERR_SEQ_LEN = 2,           /* SEQ_LEN == 0 */
    GQA_ERR_N_KV_TILES = 3,        /* N_KV_TILES != ceil(SEQ_LEN / KV_BLOCK_LEN) */
    GQA_ERR_SCALE = 4,             /* SCALE_FACTOR == 0 (or not finite) */
    GQA_ERR_QUERY_POSITION = 5,    /* QUERY_POSITION >= SEQ_LEN */
    GQA_ERR_KV_BLOCK_LEN = 6,      /* KV_BLOCK_LEN == 0 */
    GQA_ERR_GROUP_SIZE = 7,        /* GROUP_SIZE != N_Q_HEADS / N_KV_HEADS */
    GQA_ERR_NULL_POINTER = 8,
    GQA_ERR_ALIGNMENT = 9,         /* pointer not 16-byte aligned or stride not a multiple of 8 */
    GQA_ERR_WORKSPACE = 10,        /* workspace missing or smaller than gqa_workspace_bytes() */
    GQA_ERR_BATCH = 11,            /* batch < 1, or a per-sequence descriptor is invalid */
    GQA_ERR_KV_RANGE = 12,         /* stored key range [pos_begin, pos_end) invalid */
    GQA_ERR_CUDA = 13,             /* a CUDA runtime call (launch, attribute, copy) failed */
    GQA_ERR_DEVICE_TIMEOUT = 14,   /* a bounded wait inside a kernel gave up (see gqa_read_status) */
    GQA_ERR_UNSUPPORTED_DEVICE = 15, /* current device is not sm_100 */
    GQA_ERR_ROPE_THETA = 16,       /* rope_theta <= 0, not finite, or a 5th distinct value on one device */
    GQA_ERR_FLAGS = 17,            /* gqa_params.flags holds a bit this entry point does not know */
    GQA_ERR_MEMORY = 18,           /* a tensor, table or workspace pointer is not memory of the current
                                      GPU (host memory, pageable or pinned, or another GPU's memory) */
    GQA_ERR_KV_HEADS = 19          /* KV-head range empty or outside [0, 8) (gqa_decode_heads) */
};

/* GQA_FLAG_* values for gqa_params.flags. */
#define GQA_FLAG_PARTIAL_OUT 0x1u  /* write FP32 partials (see gqa_partial_row) instead of BF16 rows */
/* K rows are stored already rotated: RoPE was applied when each row was appended
 * (gqa_rope_k_cache), so decode rotates only Q.  The production KV-cache
 * convention; with it the reference's per-call RoPE of every K row
 * (gen_gqa_wrapper_vectors.py:122-124, rope_unit.v) moves to append time.
 * Accepted by gqa_decode, gqa_decode_batched, gqa_decode_noalloc and
 * gqa_decode_exchange. */
#define GQA_FLAG_K_ROTATED 0x2u
/* Q rows are supplied already rotated at QUERY_POSITION (with
 * GQA_FLAG_K_ROTATED: the RTL-numerics mode, where both come from
 * gqa_rope_rtl).  Accepted where GQA_FLAG_K_ROTATED is. */
#define GQA_FLAG_Q_ROTATED 0x4u

/*
 * Call parameters.  The first block mirrors the reference's AXI-Lite register
 * map (axi_lite_regs.v:5-24) and RTL parameters (gqa_attention_wrapper.v:47-68);
 * the rest describes where the tensors live.  Strides are in elements.
 *
 *   Q   : q  + b*q_batch_stride + qh*q_head_stride + d
 *   K/V : k  + row*k_pos_stride + kh*k_head_stride + d,  row = kv_start + (p - pos_begin)
 *   out : out + b*out_batch_stride + qh*out_head_stride + d
 *
 * Head-major transport order ([8][KV_INPUT_LEN][128], gen_gqa_wrapper_vectors.py:116-119)
 * is k_pos_stride=128, k_head_stride=KV_INPUT_LEN*128; a position-major KV cache
 * ([S][8][128]) is k_pos_stride=1024, k_head_stride=128.
 */
typedef struct gqa_params {
    uint32_t n_q_heads;       /* 0x08 N_Q_HEADS      (must be 32)  */
    uint32_t n_kv_heads;      /* 0x0C N_KV_HEADS     (must be 8)   */
    uint32_t head_dim;        /* 0x10 HEAD_DIM       (must be 128) */
    uint32_t tile_dim;        /* 0x14 TILE_DIM       (must be 16; the AXIS beat width, no effect on layout) */
    uint32_t seq_len;         /* 0x18 SEQ_LEN        (single-sequence calls) */
    uint32_t n_kv_tiles;      /* 0x1C N_KV_TILES     (single-sequence calls) */
    float    scale;           /* 0x24 SCALE_FACTOR, as a float: the golden uses exactly 1/sqrt(128) */
    uint32_t query_position;  /* 0x28 QUERY_POSITION (single-sequence calls) */
    uint32_t kv_block_len;    /* KV_BLOCK_LEN: keys per hardware block (padding granularity) */
    uint32_t group_size;      /* GROUP_SIZE contract: N_Q_HEADS / N_KV_HEADS */
    float    rope_theta;      /* 500000 for Llama-3 */
    uint32_t flags;           /* GQA_FLAG_* */
    int64_t  q_batch_stride, q_head_stride;
    int64_t  k_pos_stride, k_head_stride;
    int64_t  v_pos_stride, v_head_stride;
    int64_t  out_batch_stride, out_head_stride;
    uint8_t *mask_out;        /* optional debug export: key_valid() per padded key position */
    int64_t  mask_stride;     /* bytes between sequences in mask_out */
} gqa_params;

/*
 * One sequence of a batched call.  The keys this call reads are the absolute
 * positions [pos_begin, pos_end) intersected with the visible set
 * [0, min(seq_len, query_position + 1)); key p is stored at row
 * kv_start + (p - pos_begin).  pos_begin=0, pos_end=seq_len is a whole
 * sequence; a sequence shard on one GPU of several uses its own sub-range.
 */
typedef struct gqa_seq_desc {
    int64_t kv_start;
    int32_t seq_len;
    int32_t query_position;
    int32_t pos_begin;
    int32_t pos_end;
} gqa_seq_desc;

/* FP32 partial result for one Q head, written with GQA_FLAG_PARTIAL_OUT:
 * acc = sum_p 2^(s_p - m) * V_p, l = sum_p 2^(s_p - m), s_p the score in log2
 * units.  A head with no keys has m = -inf, l = 0, acc = 0.  out_head_stride and
 * out_batch_stride are then in floats and must be >= 132 / >= 32*132. */
typedef struct gqa_partial_row {
    float acc[128];
    float m;
    float l;
    float pad[2];
} gqa_partial_row;

/* Message for a status code (static string). */
const char *gqa_status_string(int status);

/* Library version, (major << 16) | (minor << 8) | patch. */
int gqa_version(void);

/* 1 if `device` is an sm_100 GPU this library was compiled for, else 0. */
int gqa_device_supported(int device);

/*
 * Host-side configuration check of a single-sequence call, without touching the
 * GPU.  Replaces the START-time config_error (gqa_attention_wrapper.v:230-237)
 * and the generator's checks (gen_gqa_wrapper_vectors.py:57-78).
 */
int gqa_validate(const gqa_params *p);

/*
 * Bytes of device workspace a call needs (0 on invalid input).  `descs` is the
 * host copy of the batch's descriptors, or NULL with batch == 1 for a
 * single-sequence call described by p->seq_len / p->query_position.
 * The workspace's first 256 bytes (the device status word, the per-KV-head
 * arrival counters of the single-sequence split merge and a batch's work-queue
 * counters) must be zero when it is allocated; every call leaves the counters
 * zero again, and gqa_read_status
 * clears the whole header after a timed-out wait.  The rest needs no
 * initialisation (every call writes its split partials before reading them).
 * Calls that share a workspace must be ordered (one stream).  With `descs`
 * and batch 1 the size also covers gqa_decode_exchange of that shard.
 */
size_t gqa_workspace_bytes(const gqa_params *p, const gqa_seq_desc *descs, int batch);

/*
 * Diagnostic (no reference counterpart): how a call on the current device cuts
 * the keys.  `descs`/`batch` as for gqa_workspace_bytes.  Writes the total
 * number of key splits, the keys per split, and the cluster size (> 0 when a
 * single sequence's splits of each KV head run as one thread-block cluster and
 * merge on chip; 0 when the last split of each KV head to finish merges them
 * (one sequence, also a batched call of one) or split_merge_kernel does
 * (batched call of several).  Returns a status.
 */
int gqa_decode_plan(const gqa_params *p, const gqa_seq_desc *descs, int batch, int *splits, int *keys_per_split,
                    int *cluster);

/*
 * Host-only planning (no reference counterpart): the split plan of a call on a
 * GPU with `sms` SMs, computed without any CUDA call or device.  `descs`/`batch`
 * as for gqa_workspace_bytes.  Thread-block clusters are left out, so the result
 * equals gqa_decode_plan's on such a GPU whenever that reports cluster 0, as it
 * does for every batch of several sequences and for long single sequences (on
 * the B200s measured, for instance, SEQ_LEN 4096 and 131072).  For a scheduler
 * that sizes work before it holds a GPU, and for tests of the planner on
 * machines without one.  Writes the total
 * number of key splits (each runs on 8 CTAs, one per KV head) and the keys per
 * split.  Returns a status (GQA_ERR_BATCH for sms < 1).
 */
int gqa_decode_plan_host(const gqa_params *p, const gqa_seq_desc *descs, int batch, int sms, int *splits,
                         int *keys_per_split);

/*
 * Single-token decode of one sequence: the operation the reference performs
 * between START (axi_lite_regs.v:147-151) and the last output row
 * (gqa_attention_wrapper.v:186-222); numerically the golden of
 * pyfiles/gen_gqa_wrapper_vectors.py:121-139.
 * q: [32][128] BF16; k, v: the key/value rows (layout from the strides);
 * out: [32][128] BF16 (or gqa_partial_row[32] with GQA_FLAG_PARTIAL_OUT).
 * The first call on a device with a given rope_theta uploads that theta's
 * RoPE table (a synchronous copy; make it before any stream capture); up to 4
 * distinct rope_theta values per device.
 */
int gqa_decode(const void *q, const void *k, const void *v, void *out,
               const gqa_params *p, void *workspace, size_t workspace_bytes, void *stream);

/*
 * gqa_decode of the KV heads [kv_head_begin, kv_head_begin + kv_head_count)
 * only, and of their Q heads 4h .. 4h+3 (the GQA mapping of
 * gqa_controller.v:159-162: a KV head and its Q group depend on no other head).
 * For a sequence whose KV heads are sharded across GPUs: each GPU holds the K/V
 * rows of its heads only and decodes them with the whole GPU, with no exchange.
 *  - k, v: kv_head_count heads (head index h - kv_head_begin in the strides).
 *  - q, out: the full 32-head layout; only the range's Q rows are read and only
 *    its output rows written.
 *  - workspace: gqa_workspace_bytes_heads(p, kv_head_count) bytes, header
 *    zeroed as for gqa_decode.
 * Returns GQA_ERR_KV_HEADS for an empty range or one outside [0, 8).
 */
size_t gqa_workspace_bytes_heads(const gqa_params *p, int kv_head_count);
int gqa_decode_heads(const void *q, const void *k, const void *v, void *out, const gqa_params *p,
                     int kv_head_begin, int kv_head_count, void *workspace, size_t workspace_bytes, void *stream);

/*
 * gqa_decode without a workspace argument: no counterpart in the reference.
 * For callers that may not allocate device memory (a plug-in inside a host
 * program that owns every device allocation, or a loop that cannot afford
 * cudaMalloc's implicit synchronisation), the split table and partials live in
 * a library-owned device array of GQA_NOALLOC_SCRATCH_BYTES; each GPU that
 * loads the library holds that array until the process exits.  Nothing is
 * allocated or freed by this call.
 *  - The first call on a device looks up the array's device address for that
 *    device (cudaGetSymbolAddress), and the first call on a device with a
 *    given rope_theta uploads that theta's RoPE table with a synchronous
 *    cudaMemcpy, as gqa_decode does: such a first call synchronises the
 *    device.  Make it before any stream capture begins and outside
 *    latency-critical loops; later calls synchronise nothing.
 *  - The address is kept for the life of the process: after a
 *    cudaDeviceReset on a device that has used this entry point, do not call
 *    it again on that device.
 *  - A call whose scratch would exceed GQA_NOALLOC_SCRATCH_BYTES returns
 *    GQA_ERR_WORKSPACE without launching; use gqa_decode with a workspace.
 *    A single sequence is cut into at most one wave of splits (8 CTAs each)
 *    and at most 32 splits, so it needs at most 512 + min(SMs / 8, 32) x
 *    16,896 bytes: 0.3 MiB on a 148-SM B200, 0.54 MiB on any GPU, so this
 *    refusal is a guard that valid calls do not reach.
 *  - All calls on a device share the one array and it keeps the last call's
 *    contents: calls whose kernels overlap on the GPU (several streams, or
 *    several host threads) race and corrupt each other's results; serialise
 *    them.  In-kernel wait timeouts are not reported on this path.
 */
#define GQA_NOALLOC_SCRATCH_BYTES ((size_t)1 << 20)
int gqa_decode_noalloc(const void *q, const void *k, const void *v, void *out,
                       const gqa_params *p, void *stream);

/*
 * Batched (ragged) decode: one query token per sequence, B sequences.  The
 * per-sequence register values come from `descs`; `host_descs` is the same
 * array in host memory (used to validate and plan), `dev_descs` in device
 * memory (read by the kernel).  p->seq_len / n_kv_tiles / query_position are
 * ignored.  The reference handles one sequence per START (gqa_controller.v:140-277);
 * this entry point runs B of them in one launch.
 */
int gqa_decode_batched(const void *q, const void *k, const void *v, void *out,
                       const gqa_params *p, const gqa_seq_desc *host_descs,
                       const gqa_seq_desc *dev_descs, int batch,
                       void *workspace, size_t workspace_bytes, void *stream);

/*
 * Log-sum-exp combine of `n_parts` FP32 partial results (gqa_partial_row) into
 * BF16 rows: out = sum_s 2^(m_s-M) acc_s / sum_s 2^(m_s-M) l_s with M = max_s m_s.
 * This is the rescale-and-normalise of flash_softmax.v:233-512 and
 * output_accumulator.v:398-687 applied across sequence shards.
 * partials: part s, sequence b, head h at partials + s*part_stride + b*batch_stride + h*132 floats.
 */
int gqa_combine_partials(const float *partials, int n_parts, int64_t part_stride,
                         int64_t batch_stride, int batch, void *out,
                         int64_t out_batch_stride, int64_t out_head_stride, void *stream);

/*
 * Chunked multi-query decode (tensor cores).  For each of `batch` sequences,
 * n_queries (1..128) consecutive query positions first_position ..
 * first_position + n_queries - 1, each answered exactly as a gqa_decode call
 * with QUERY_POSITION = that position and SEQ_LEN = p->seq_len (the
 * equivalence "128 sequential single-position calls" of the reference's
 * chunked configuration, gen_gqa_wrapper_vectors.py:121-139 per query).
 *
 *   Q   : q + b*p->q_batch_stride + i*q_query_stride + qh*p->q_head_stride + d
 *   K/V : k + b*k_batch_stride + pos*p->k_pos_stride + kh*p->k_head_stride + d
 *   out : out + b*p->out_batch_stride + i*out_query_stride + qh*p->out_head_stride + d
 *
 * p is validated as gqa_validate does with QUERY_POSITION = the last query's
 * position; p->flags must be 0 and p->mask_out NULL.  The workspace needs at
 * least GQA_CHUNKED_WORKSPACE_BYTES bytes whose first 256 are zero (the device
 * status word, read with gqa_read_status).  With gqa_chunked_workspace_bytes()
 * bytes the call also splits the (sequence, Q head) units of the last, partly
 * filled wave of CTAs along the keys to fill it, and merges their parts with a
 * second small kernel; with fewer it runs every unit whole.  No reference
 * counterpart beyond the per-query golden: the RTL decodes one position per START.
 */
typedef struct gqa_chunk_params {
    uint32_t batch;
    uint32_t n_queries;
    uint32_t first_position;
    uint32_t reserved;          /* must be 0 */
    int64_t  q_query_stride;    /* elements between consecutive queries of a sequence */
    int64_t  out_query_stride;
    int64_t  k_batch_stride;    /* elements between sequences in K and in V */
    int64_t  v_batch_stride;
} gqa_chunk_params;

#define GQA_CHUNKED_WORKSPACE_BYTES ((size_t)256)

/* Workspace for gqa_decode_chunked with the key-range split of the last wave
 * (on the current device); 0 on invalid input. */
size_t gqa_chunked_workspace_bytes(const gqa_params *p, const gqa_chunk_params *c);

int gqa_decode_chunked(const void *q, const void *k, const void *v, void *out, const gqa_params *p,
                       const gqa_chunk_params *c, void *workspace, size_t workspace_bytes, void *stream);

/*
 * RoPE of `rows` 128-element BF16 rows, row r at positions[r], to FP32 rows:
 * the rotation of rope_unit.v / rope_half_split (gen_gqa_wrapper_vectors.py:25-35)
 * with the same device code the decode kernel uses.
 */
int gqa_rope_rows(const void *x, const int32_t *positions, float *out, int rows,
                  float rope_theta, void *stream);

/*
 * Pre-rotated K cache: RoPE of the K rows of `n_positions` positions, 8 KV
 * heads each, written as BF16 (round to nearest even).  Row (i, h) is
 * k + i*pos_stride + h*head_stride (elements) and turns by positions[i]
 * (rope_half_split, gen_gqa_wrapper_vectors.py:25-35, with exact per-element
 * factors).  k_rot has the same layout; k_rot == k rotates in place.  Decode
 * such a cache with GQA_FLAG_K_ROTATED.  Pointers 16-byte aligned, strides
 * multiples of 8.
 */
int gqa_rope_k_cache(const void *k, void *k_rot, const int32_t *positions, int n_positions,
                     int64_t pos_stride, int64_t head_stride, float rope_theta, void *stream);

/*
 * RTL-numerics RoPE (rope_unit.v): rows rotated the way the reference RTL
 * does, for comparing against a dump of its datapath.  Pair i of a row at
 * position p turns by the ROM entry at the top `rom_addr_bits` bits of the
 * 32-bit phase (phase_rom[i] * p) mod 2^32 (rope_unit.v:159-172), and the
 * rotation runs through BF16 multiply and add/subtract units
 * (rope_unit.v:124-129), each rounding its exact result to BF16 as the
 * reference defines them (gen_bf16_primitive_vectors.py:31-32).
 * Rows: `heads` per position, row (i, h) at x + i*pos_stride + h*head_stride
 * (elements), turned by positions[i]; `out` has the same layout (in place
 * allowed).  phase_rom (head_dim/2 words) and sincos_rom (2^rom_addr_bits
 * words, {cos_bf16 << 16 | sin_bf16}) are in device memory: the tables of
 * gqa_rope_phase_rom / gqa_rope_sincos_rom (tools/gen_rope_rom.py).
 * Decode the rotated Q and K with GQA_FLAG_Q_ROTATED | GQA_FLAG_K_ROTATED and
 * the BF16 scale register value (0x3DB5 for head_dim 128) as `scale`.
 */
int gqa_rope_rtl(const void *x, void *out, const int32_t *positions, int n_positions, int heads,
                 int64_t pos_stride, int64_t head_stride, const uint32_t *phase_rom,
                 const uint32_t *sincos_rom, int rom_addr_bits, void *stream);

/*
 * The RoPE ROM tables of tools/gen_rope_rom.py:41-57, computed on the host:
 * phase[i] = round(theta^(-i/(head_dim/2)) * 2^32 / 2pi) mod 2^32 (head_dim/2 entries);
 * sincos[a] = (bf16(cos 2pi a/N) << 16) | bf16(sin 2pi a/N), N = 2^addr_bits.
 */
int gqa_rope_phase_rom(uint32_t *phase, int head_dim, double rope_theta);
int gqa_rope_sincos_rom(uint32_t *sincos, int addr_bits);

/*
 * Long-context sequence split across the GPUs of one node: exchange of the
 * per-GPU FP32 partial rows (GQA_FLAG_PARTIAL_OUT) over NVLink peer memory,
 * fused with the log-sum-exp combine (no collective library).  Each rank
 * creates one exchange buffer, shares its CUDA IPC handle with the other ranks
 * (e.g. over torch.distributed), opens theirs, and passes a DEVICE array of all
 * `world` buffer pointers (its own at index `rank`) to gqa_combine_peers, which
 * publishes this rank's partials, waits (bounded, ~1 s) for every peer's, and
 * writes the merged BF16 rows [batch][32][128] on every rank.  Calls must be
 * made in the same order on all ranks; the exchange epoch lives in the buffer,
 * so CUDA-graph replays work.  A timed-out wait sets the workspace status word
 * (gqa_read_status); the exchange must then be re-created.  batch <= 64 (all
 * CTAs of the exchange resident at once).  No reference counterpart: the
 * reference has one device.
 */
#define GQA_PEER_HANDLE_BYTES 64
size_t gqa_peer_buffer_bytes(int batch);
int gqa_peer_buffer_create(size_t bytes, void **buffer, void *ipc_handle);
int gqa_peer_buffer_open(const void *ipc_handle, void **buffer);
int gqa_peer_buffer_close(void *buffer);
int gqa_peer_buffer_destroy(void *buffer);
int gqa_combine_peers(const float *partials, int64_t partial_batch_stride, const void *const *peer_buffers,
                      int world, int rank, int batch, void *out, int64_t out_batch_stride,
                      int64_t out_head_stride, void *workspace, void *stream);

/*
 * The same exchange fused into the decode kernel: this rank decodes its shard
 * `shard` (pos_begin/pos_end of one sequence, as for gqa_decode_batched with
 * batch 1), and the CTA that merges each KV head's splits publishes the head's
 * rows to the exchange buffer, waits for the peers' rows over NVLink and writes
 * the final BF16 rows of the whole sequence to `out` [32][128] on every rank —
 * one launch per step, no combine kernel.  The rows are pushed into every
 * rank's buffer as 64-bit words that carry the step's epoch beside each value,
 * and each rank waits (bounded) on those words in its own memory.
 * 2 <= world <= 8.
 * `workspace`: gqa_workspace_bytes(p, shard, 1) bytes (the 256-byte header zeroed
 * at allocation).  p->flags must be 0.  The exchange buffers are those of
 * gqa_peer_buffer_create (batch 1).
 */
int gqa_decode_exchange(const void *q, const void *k, const void *v, void *out, const gqa_params *p,
                        const gqa_seq_desc *shard, const void *const *peer_buffers, int world, int rank,
                        void *workspace, size_t workspace_bytes, void *stream);

/*
 * Read (and clear) the device status word a kernel leaves in `workspace`:
 * GQA_OK, or GQA_ERR_DEVICE_TIMEOUT if a bounded wait gave up.  Synchronises
 * `stream`.  Plays the part of ERROR_FLAGS/STATUS (axi_lite_regs.v:153-157,178).
 */
int gqa_read_status(void *workspace, void *stream, int *device_status);

/* ---------------------------------------------------------------------------
 * The ".mem" transport text on the GPU.  Replaces the reference's host codec
 * pyfiles/gqa_reference.py:26-46 (pack_bf16, unpack_bf16, write_mem, read_mem)
 * for the vectors of gen_gqa_wrapper_vectors.py:111-119.
 *
 * A line holds `elements` BF16 codes as 4*elements hex digits, element 0 in
 * the rightmost 4.  Decoding follows read_mem: lines end at \n, \r, \r\n, \v,
 * \f or \x1c-\x1e; blank lines and lines whose first non-blank characters are
 * "//" are skipped; '_' is ignored; blanks (space, \t, \x1f) may surround the
 * digits but not sit between them; any other byte, or a digit count other
 * than 4*elements, makes the line malformed.
 * ------------------------------------------------------------------------- */
#define GQA_MEM_MAX_ELEMENTS 4096

typedef struct gqa_mem_result {
    uint64_t rows;       /* data lines found (valid or malformed) */
    uint64_t bad_offset; /* byte offset of the first malformed line, UINT64_MAX if none */
} gqa_mem_result;

/* Scratch for gqa_mem_decode: 8 bytes per 16 KB of text. */
size_t gqa_mem_decode_workspace_bytes(size_t text_bytes);

/*
 * Decode `text` (device memory, 16-byte aligned, text_bytes long) into `rows`
 * (device, uint16 [max_rows][elements], 4-byte aligned).  Rows past max_rows
 * are counted but not written.  `result` (device memory) receives the row
 * count and the first malformed line; read it after the stream has passed
 * this call: the decode is valid iff result.bad_offset == UINT64_MAX and
 * result.rows <= max_rows.  Asynchronous on `stream`; three kernel launches.
 */
int gqa_mem_decode(const void *text, size_t text_bytes, int elements, void *rows, uint64_t max_rows,
                   gqa_mem_result *result, void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of text gqa_mem_encode writes: n_rows * (4*elements + 1). */
size_t gqa_mem_encode_bytes(uint64_t n_rows, int elements);

/*
 * Encode `rows` (device, uint16 [n_rows][elements]) as write_mem's text:
 * lowercase hex, element 0 rightmost, '\n' after every line (the trailing
 * newline included).  `text` (device, 16-byte aligned) receives
 * gqa_mem_encode_bytes(n_rows, elements) bytes.  Asynchronous on `stream`.
 */
int gqa_mem_encode(const void *rows, uint64_t n_rows, int elements, void *text, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GQA_B200_H */
