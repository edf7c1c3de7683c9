/*
 * qcc_b200.h -- C ABI of the B200 indexed sparse gated-FFN engine.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * launches on that stream, never synchronises and never allocates memory.
 * Scratch memory is caller-provided ("workspace"); its size is given by the
 * matching *_workspace_bytes() query and it must be zero-filled once with
 * qcc_workspace_init() before first use (each call leaves its counters at
 * zero again).  A workspace must not be shared by calls that can overlap on
 * the GPU.
 *
 * Return value: QCC_OK (0) or one of the QCC_ERR_* host-side codes below.
 * Conditions that are only visible on the device (an index out of range, a
 * bounded wait that ran out) are recorded as QCC_DEV_* bits in the status
 * word at the start of the workspace; qcc_workspace_status_offset() gives
 * its byte offset so a caller can read it back when it chooses to sync.
 *
 * Packed weight layout (neuron-major, one record per intermediate neuron n):
 *     record n = [ gate[n, 0:Hp] | up[n, 0:Hp] | down[0:Hp, n] ]
 * with Hp = hidden rounded up to a multiple of 8 elements, zero padded, and record stride 3 * Hp * sizeof(dtype) bytes (30720 B for
 * hidden = 5120 bf16).  The reference keeps gate [N,H], up [N,H] and
 * down [H,N] as separate tensors (runtime/weights.py:89-96 writes only a
 * separate transposed down); the interleaved record is new and lets one bulk
 * copy fetch everything a selected neuron needs.
 */
#ifndef QCC_B200_H
#define QCC_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define QCC_API __attribute__((visibility("default")))
#else
#define QCC_API
#endif

#define QCC_ABI_VERSION 2

/* Element types (weights, x, y, activations). */
#define QCC_DTYPE_BF16 0
#define QCC_DTYPE_F16 1
#define QCC_DTYPE_F32 2
/* Index types. */
#define QCC_INDEX_I32 0
#define QCC_INDEX_I64 1
/* Flag OR-ed into the index type of the decode entry points: the ids (and
 * n_ids_dev / token_mask, when given) are not written by any qcc_* kernel
 * launched earlier on the same stream -- e.g. they came from a host copy or
 * from another library's kernel.  The decode kernels let the next launch on
 * the stream start before they finish; with this flag a decode launch reads
 * its ids and starts its record copies at once, while the launches ahead of
 * it are still finishing, and waits for them only before it reads x.  Do not
 * set it for ids produced by qcc_select_topk, qcc_build_union or
 * qcc_selector_scores_topk on the same stream. */
#define QCC_IDS_READY 0x100

/* OR-ed into the index type of the decode entry points, QCC_MASK_SHIFT(s),
 * s in 0..7: token b of the call uses bit s + b of each token_mask byte (and
 * s + batch <= 8).  A host that splits a batch of up to 8 tokens into calls of
 * qcc_decode_max_batch tokens passes the same mask with the chunk's first token
 * as s instead of a shifted copy. */
#define QCC_MASK_SHIFT(s) (((s) & 7) << 12)

/* Host-side status codes. */
#define QCC_OK 0
#define QCC_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad enum */
#define QCC_ERR_SHAPE 2            /* inconsistent sizes / strides            */
#define QCC_ERR_DTYPE 3            /* unsupported dtype combination           */
#define QCC_ERR_ALIGNMENT 4        /* pointer or stride not 16-byte aligned   */
#define QCC_ERR_UNSUPPORTED 5      /* size beyond what the kernels handle     */
#define QCC_ERR_WORKSPACE 6        /* workspace missing or too small          */
#define QCC_ERR_CUDA 7             /* a CUDA runtime call or launch failed    */

/* Device-side status bits (sticky, OR-ed into the workspace status word). */
#define QCC_DEV_ID_RANGE 1u /* a selected id was outside [0, n_records)      */
#define QCC_DEV_TIMEOUT 2u  /* a bounded wait on a bulk copy ran out          */

/* Library version (QCC_ABI_VERSION). */
QCC_API int qcc_version(void);

/* Human-readable text for a QCC_ERR_* code (static storage). */
QCC_API const char* qcc_status_string(int status);

/* Text of the last CUDA error seen by this library on the calling thread. */
QCC_API const char* qcc_last_cuda_error_string(void);

/* Padded segment length Hp for a hidden size and dtype. */
QCC_API int qcc_hidden_pad(int hidden, int dtype);

/* Record stride in bytes: 3 * Hp * sizeof(dtype). */
QCC_API int64_t qcc_record_bytes(int hidden, int dtype);

/* ---------------------------------------------------------------------- */
/* Packing                                                                 */
/* ---------------------------------------------------------------------- */

/*
 * Build the neuron-major packed array from the reference's three tensors.
 * Replaces the layout step of runtime/weights.py:89-96
 * (save_neuron_major_layout) and the per-call gathers of
 * runtime/ffn.py:20-23 (gather_weights): the gathers become one bulk copy
 * per selected record inside qcc_indexed_ffn_decode.
 *   gate, up : [n_records, hidden] row-major, row stride ld_gu elements
 *   down     : element (h, n) at down[h * down_stride_h + n * down_stride_n]
 *              ([hidden, n_records] row-major: (n_records, 1); the
 *              reference's transposed down_t [n_records, hidden]: (1, hidden))
 *   packed   : [n_records, 3 * Hp] (stride qcc_record_bytes)
 */
QCC_API int qcc_pack_records(const void* gate, const void* up, int64_t ld_gu, const void* down,
                             int64_t down_stride_h, int64_t down_stride_n, int64_t n_records, int hidden, int dtype,
                             void* packed, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Fused indexed gated FFN (decode / small batch)                          */
/* ---------------------------------------------------------------------- */

/* Largest batch one qcc_indexed_ffn_decode call accepts (the same bound
 * holds for qcc_ffn_activations and qcc_indexed_ffn_down).  bf16 / fp16
 * records whose hidden size rounded up to 8 is a multiple of 128 run 2 or
 * more tokens on the tensor cores: 8 up to hidden 6144, 6 up to 8192, 4 up
 * to 10240.  Otherwise (fp32, other sizes) 4 for hidden <= 5120 and 1 for
 * hidden <= 10240; 0 beyond 10240. */
QCC_API int qcc_decode_max_batch(int hidden, int dtype);

/* Bytes of workspace qcc_indexed_ffn_decode needs for this batch/hidden. */
QCC_API size_t qcc_decode_workspace_bytes(int batch, int hidden, int dtype);

/* Byte offset of the device status word inside any qcc workspace (0). */
QCC_API size_t qcc_workspace_status_offset(void);

/* Zero-fill a workspace on `stream` (cudaMemsetAsync; allocates nothing). */
QCC_API int qcc_workspace_init(void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * y[b, :] = sum_j  m[j,b] * silu(G[id_j] . x[b]) * (U[id_j] . x[b]) * D[:, id_j]
 * for the selected records id_j, j < n_ids.
 *
 * Replaces runtime/cuda_indexed.py:61-64 (cuda_indexed_ffn ->
 * indexed_ffn_cuda, two launches: gate_up then down) and
 * runtime/ffn.py:34-39 (TorchDynamicSparseFFN.forward).  Math follows
 * runtime/ffn.py:26-31: activation = silu(gate) * up, y = activation @ down.
 * Accumulation is fp32 throughout; y is rounded once to y_dtype.
 * Two launches on `stream`: the record stream (one CTA per SM, each storing
 * a partial y row in the workspace) and a reduce of those rows in a fixed
 * order, so y is bit-reproducible for a given device.  Both let the next
 * launch on the stream be scheduled early (programmatic dependent launch).
 *
 *   x          : [batch, hidden] in `dtype`, row stride ldx elements
 *   packed     : qcc_pack_records layout, n_records records
 *   ids        : n_ids selected record indices (ids_dtype QCC_INDEX_I32 or
 *                _I64, optionally | QCC_IDS_READY | QCC_MASK_SHIFT(s)); any
 *                order, duplicates
 *                count twice (as index_select does); out-of-range ids
 *                contribute nothing and raise QCC_DEV_ID_RANGE
 *   n_ids_dev  : optional device int32 count; when non-null the kernel uses
 *                min(*n_ids_dev, n_ids) ids (output of qcc_build_union)
 *   token_mask : optional [n_ids] bytes; bit b set = token b uses record j
 *                (bit s + b with QCC_MASK_SHIFT(s) in ids_dtype).  Null
 *                means every token uses every record (the reference's one
 *                shared 1-D id list, runtime/ffn.py:20-23).
 *   y_out      : [batch, hidden] in y_dtype (dtype or QCC_DTYPE_F32)
 *   y_in       : optional fp32 [batch, hidden] (row stride ld_in) added to
 *                the sum before the final rounding: a residual, or the
 *                partial result of an earlier call over other records
 *   activation_out : optional [batch, n_ids] in `dtype`, the per-record
 *                activation (cuda_indexed_parts' first result,
 *                runtime/cuda_indexed.py:56-59); entries of records a token
 *                does not use are 0.
 * batch must be 1..qcc_decode_max_batch(hidden, dtype) per call (a host
 * wrapper chunks larger batches).
 */
QCC_API int qcc_indexed_ffn_decode(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                   int64_t n_records, int dtype, const void* ids, int ids_dtype, int n_ids,
                                   const int32_t* n_ids_dev, const uint8_t* token_mask, void* workspace,
                                   size_t workspace_bytes, void* y_out, int64_t ldy, int y_dtype, const float* y_in,
                                   int64_t ld_in, void* activation_out, int64_t lda, cudaStream_t stream);

/*
 * Gate / up pass of the oracle-mode FFN: for every record n < n_records (all
 * of them, in order) and token b < batch,
 *   act_out[b * ld_act + n]       = silu(G[n] . x[b]) * (U[n] . x[b])   (fp32)
 *   scores_out[b * ld_scores + n] = |act| * col_weights[n] (|act| when
 *                                   col_weights is NULL; scores_out may be NULL)
 * streaming only the gate and up parts of each record (2/3 of it).  The
 * reference computes this activation with the model's dense gate and up
 * projections and scores it in end_to_end/oracle_sparse_mlp.py:64-75
 * (|a| * ||down column||) or oracle/importance.py:10-13 (|a|).  batch <=
 * qcc_decode_max_batch; the workspace is the decode workspace (its status
 * word reports QCC_DEV_TIMEOUT).  One launch; fp32 arithmetic.
 */
QCC_API int qcc_ffn_activations(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                int64_t n_records, int dtype, const float* col_weights, float* act_out, int64_t ld_act,
                                float* scores_out, int64_t ld_scores, void* workspace, size_t workspace_bytes,
                                cudaStream_t stream);

/*
 * Down pass of the oracle-mode FFN: y[b] = sum_j m[j,b] * act[b * ld_act + id_j] * D[:, id_j]
 * (+ y_in) for the selected records id_j, streaming only the down part of
 * each selected record (1/3 of it).  act is the activation of every record
 * (act_dtype: bf16, fp16 or fp32), as qcc_ffn_activations writes it, indexed
 * by record id; ids, n_ids_dev and token_mask as in qcc_indexed_ffn_decode
 * (the output of qcc_build_union for per-token selections).  Replaces the
 * scatter into zeros and the dense down projection of
 * end_to_end/oracle_sparse_mlp.py:75 and oracle/sparse_ffn.py:8-13.  Same two
 * launches, workspace and determinism as qcc_indexed_ffn_decode.
 */
QCC_API int qcc_indexed_ffn_down(const void* act, int64_t ld_act, int act_dtype, int batch, int hidden,
                                 const void* packed, int64_t n_records, int dtype, const void* ids, int ids_dtype,
                                 int n_ids, const int32_t* n_ids_dev, const uint8_t* token_mask, void* workspace,
                                 size_t workspace_bytes, void* y_out, int64_t ldy, int y_dtype, const float* y_in,
                                 int64_t ld_in, cudaStream_t stream);

/* Bytes of the scratch built into the library for
 * qcc_indexed_ffn_decode_static (4 MiB). */
#define QCC_STATIC_SCRATCH_BYTES (4u << 20)

/*
 * qcc_indexed_ffn_decode without a workspace argument; it reports no device
 * status (QCC_DEV_* bits are not readable), so out-of-range ids and bounded
 * waits that ran out go unseen, although out-of-range ids still contribute
 * nothing.  For callers that cannot allocate device memory where they run
 * the layer: code inside another framework's allocator or memory pool,
 * plugin hosts that only hand over the input and output buffers, loops that
 * must not call cudaMalloc / cudaFree because those can synchronise the
 * device.  No counterpart in the reference, whose extension allocates its
 * outputs per call.
 *
 * Otherwise the same arguments and results as qcc_indexed_ffn_decode minus
 * the workspace (and without the y_in input).  The scratch is a fixed
 * QCC_STATIC_SCRATCH_BYTES array in the library image, held by every GPU that
 * loads the library until the process exits; requests needing more
 * (qcc_decode_workspace_bytes(batch, hidden, dtype) larger than that: one
 * token up to hidden 6552) return QCC_ERR_WORKSPACE.  The call allocates
 * nothing.  The first call on each device looks the scratch up with
 * cudaGetSymbolAddress (which may load the module there), so make it before
 * any stream capture; the address is kept for the life of the process, so a
 * cudaDeviceReset (or any other teardown of the device's primary context)
 * makes this entry point unusable on that device.  Nothing in the scratch
 * needs clearing between calls (single-device decode reads no counter), but
 * all calls on a device share it: calls that can overlap on the GPU race and
 * must be serialised by the caller.
 */
QCC_API int qcc_indexed_ffn_decode_static(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                          int64_t n_records, int dtype, const void* ids, int ids_dtype, int n_ids,
                                          const int32_t* n_ids_dev, const uint8_t* token_mask, void* y_out,
                                          int64_t ldy, int y_dtype, void* activation_out, int64_t lda,
                                          cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Selector                                                                */
/* ---------------------------------------------------------------------- */

/*
 * Per row b of scores [batch, n] (fp32, row stride ld_scores): the k largest
 * scores, ties broken by lower index, -0.0 == +0.0, NaN largest; written as
 * k ascending unique int32 indices to ids_out[b * ld_ids + 0..k-1].
 * Replaces torch.topk(scores, k, sorted=False) in runtime/selector.py:24,
 * runtime/cuda_selector.py:40 and end_to_end/oracle_sparse_mlp.py:75, whose
 * tie order is unspecified; this is the deterministic order
 * sort(scores, descending, stable)[:k] then ascending.
 * n * 4 bytes must fit in shared memory (n <= 52224).
 */
QCC_API int qcc_select_topk(const float* scores, int64_t ld_scores, int batch, int n, int k, int32_t* ids_out, int64_t ld_ids,
                    cudaStream_t stream);

/*
 * Per row b of an activation act [rows, n] (bf16, fp16 or fp32, row stride
 * ld_act): the k largest scores, score = |a| * col_weights[i] (fp32, one
 * rounding) or |a| when col_weights is NULL, selected with the rule of
 * qcc_select_topk, written as k ascending int32 indices to ids_out[b * ld_ids
 * ..]; when masked_out is not NULL it receives the row with every unselected
 * entry set to 0 (same dtype, row stride ld_masked).  One launch, one CTA per
 * row, the row read once.  Replaces the scoring, torch.topk and the
 * zeros().scatter_(gather) of end_to_end/oracle_sparse_mlp.py:75 (weights =
 * down-column norms) and oracle/importance.py:10 + :21-23 (no weights).
 * n * 4 bytes must fit in shared memory (n <= 52224).
 */
QCC_API int qcc_activation_topk(const void* act, int64_t ld_act, int dtype, int rows, int n, const float* col_weights,
                                int k, int32_t* ids_out, int64_t ld_ids, void* masked_out, int64_t ld_masked,
                                cudaStream_t stream);

/*
 * Block top-K per score row (reference oracle/importance.py:26-35,
 * block_topk_indices): the row's n scores are cut into ceil(n / block) blocks
 * of `block` consecutive neurons (zero past the end), each block scored by
 * the sum of its scores (fp64 in index order, rounded once to fp32), and the
 * kb = max(1, min(n_blocks, ceil(k / block))) best blocks kept -- ties to
 * the lower block, the rule of qcc_select_topk -- as kb ascending int32 block
 * ids in block_ids[b * ld_ids ..].  Block j stands for neurons
 * [j * block, min(n, (j + 1) * block)), the expansion of
 * clustering/block_layout.py:61-64.  block_sums (optional) receives the sums.
 * One launch, one CTA per row.
 */
QCC_API int qcc_block_topk(const float* scores, int64_t ld_scores, int rows, int n, int block, int k,
                           int32_t* block_ids, int64_t ld_ids, float* block_sums, int64_t ld_sums,
                           cudaStream_t stream);

/*
 * Per tile of tile_rows consecutive rows of block_ids [rows, kb]: the union
 * of the rows' block ids, ascending, appended to tile_blocks; tile t's list is
 * tile_blocks[tile_offsets[t] .. tile_offsets[t + 1]) -- the input of
 * qcc_indexed_ffn_prefill (tile_rows 128).  tile_blocks must hold
 * ceil(rows / tile_rows) * n_blocks entries; tile_offsets ceil(rows /
 * tile_rows) + 1.  Ids outside [0, n_blocks) are skipped and set
 * QCC_DEV_ID_RANGE in *status when status is not NULL.  One CTA;
 * n_blocks <= 32768.
 */
QCC_API int qcc_tile_block_union(const int32_t* block_ids, int64_t ld_ids, int rows, int kb, int tile_rows,
                                 int n_blocks, int32_t* tile_blocks, int32_t* tile_offsets, int32_t* status,
                                 cudaStream_t stream);

/*
 * Union of the per-token sorted id lists ids [batch, k] restricted to
 * [id_begin, id_end), rebased to id_begin: union_ids gets the sorted
 * distinct local ids, token_mask bit b says token b selected it, and
 * *count_out (device int32) receives their number.  Capacity of union_ids
 * and token_mask: min(id_end - id_begin, batch * k).  batch <= 8.
 * Used for batched decode with per-token selections and for the
 * intermediate-dimension shard of each rank.  No reference counterpart
 * (the reference runs batch 1 with one id list, bridge.py:161-176).
 */
QCC_API int qcc_build_union(const int32_t* ids, int64_t ld_ids, int batch, int k, int32_t id_begin, int32_t id_end,
                    int32_t* union_ids, uint8_t* token_mask, int32_t* count_out, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Host-offload stager                                                     */
/* ---------------------------------------------------------------------- */

/*
 * Device-side neuron cache policy for one decode step of one layer whose
 * records live partly in HBM and partly in a pinned host store.  The HBM
 * "resident" array holds n_hot always-resident records in slots [0, n_hot)
 * followed by `capacity` cache slots; slot_of[n] is record n's resident slot
 * or -1.  For the step's sorted, unique ids (count k, or *k_dev when non-null)
 * it writes the resident slots of hot records and cache hits
 * (resident_out), and gives every miss the least recently used cache slot
 * this step does not use -- empty slots first, ties by the held record's id,
 * the eviction order of reference runtime/temporal.py:57-75 -- updating
 * slot_of, cache_owner, cache_last_use and lru_order in place (miss_slot_out:
 * the slots, miss_src_out: the records' cold_index entries).  lru_order
 * [capacity] lists the cache slots from least to most recently used;
 * initialise it to 0 .. capacity - 1 (with cache_owner = -1).  counts_out
 * (device int32 [6]): resident, misses served, cache hits, evicted, hot hits,
 * 1 if misses exceeded the free slots.  k <= 16384, capacity <= 8192,
 * n_records and step < 2^24 - 1.
 * One CTA; no host round trip.  The reference stages whole layers
 * synchronously (integration/freetoken_qcc/low_vram/staging.py:43-67) and
 * keeps its LRU only as a host-side simulation.
 */
QCC_API int qcc_cache_resolve(const int32_t* ids, int k, const int32_t* k_dev, int32_t* slot_of, int n_records,
                              int n_hot, int32_t* cache_owner, int32_t* cache_last_use, int32_t* lru_order,
                              int capacity, const int32_t* cold_index, int step, int32_t* resident_out,
                              int32_t* miss_slot_out, int32_t* miss_src_out, int32_t* counts_out, cudaStream_t stream);

/*
 * Copies records src_index[i] of a host store (page-locked host memory, read
 * through its device mapping; pageable memory returns
 * QCC_ERR_INVALID_ARGUMENT) into resident slots dst_slot[i] of `packed`,
 * for i < min(*count_dev, max_count) (max_count when count_dev is null).
 * Reads the host memory in place over PCIe; runs on `stream`, typically a
 * side stream overlapping the decode of the resident records.  Replaces the
 * row gather HostLayer.neuron_tensor
 * (integration/freetoken_qcc/low_vram/host_store.py:24-26) plus its copy.
 */
QCC_API int qcc_gather_records(const void* host_store, int64_t record_bytes, const int32_t* src_index,
                               const int32_t* dst_slot, const int32_t* count_dev, int max_count, void* packed,
                               cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Cross-rank sum fused into the decode (intermediate-dimension shards)    */
/* ---------------------------------------------------------------------- */

#define QCC_IPC_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer (a 256-byte header holding the
 * buffer's launch counter and its wait bound, then three rotating slots of
 * column sums for every rank) for world ranks, batch tokens and this hidden
 * size.  Size every rank's buffer for the largest batch it will serve: the
 * slots are spaced by the buffer's size, so every rank's buffer must have the
 * same size, and calls with smaller batches use the front of each slot. */
QCC_API size_t qcc_exchange_bytes(int world, int batch, int hidden, int dtype);

/* Setup-time helpers (these allocate / map, unlike every compute entry):
 * an exchange buffer initialised for use (counter zero, every column-sum word
 * the empty mark, the bits of -0.0f; synchronises the device), its CUDA IPC handle
 * (QCC_IPC_HANDLE_BYTES bytes), and the mapping of another process's buffer
 * from its handle. */
QCC_API int qcc_exchange_alloc(size_t bytes, void** ptr);
/* Re-initialise an exchange buffer in place (counter and wait bound zero,
 * every column-sum word the empty mark; synchronises the device): the
 * recovery after a QCC_DEV_TIMEOUT, done by every rank, with no call of the
 * cross-rank sum in flight on any rank, before any rank's next call. */
QCC_API int qcc_exchange_init(void* ptr, size_t bytes);
QCC_API int qcc_exchange_free(void* ptr);
QCC_API int qcc_ipc_handle(void* ptr, void* handle);
QCC_API int qcc_ipc_open(const void* handle, void** ptr);
QCC_API int qcc_ipc_close(void* ptr);
/* Bound, in ns, on each wait of the cross-rank sum for the sums of the other
 * ranks in this rank's buffer (0 = the default 2 s).  Setup time: a
 * synchronous copy into the buffer's header. */
QCC_API int qcc_exchange_set_wait_limit(void* ptr, uint64_t limit_ns);

/*
 * qcc_indexed_ffn_decode on this rank's record shard with the sum over the
 * world ranks fused into its epilogue: y_out (on every rank) =
 *   sum over ranks q in rank order of rank q's partial, + y_in.
 * id_begin >= 0: ids is the GLOBAL ascending id list shared by the batch's
 * tokens, and this rank uses the ids in [id_begin, id_end) rebased by
 * id_begin (packed holds records id_begin..id_end-1); the kernel finds that
 * run itself, so no separate union / rebase launch precedes it.  id_begin < 0:
 * ids are already local to packed (e.g. from qcc_build_union with a token
 * mask).  world 1 is allowed (no exchange; exchange may be NULL).  packed may
 * be NULL when n_records is 0 (an empty shard).
 * exchange: host array of the world ranks' exchange buffers (exchange[rank]
 * is this rank's own; the others are peer mappings from qcc_ipc_open),
 * each exchange_bytes large and initialised by qcc_exchange_alloc.  Every
 * rank makes the same sequence of calls on its buffer (the buffer counts its
 * launches; call e uses slot e % 3).  Each CTA of the reduce launch stores
 * its column sums into every rank's buffer with relaxed system-scope 16-byte
 * stores over NVLink; the words themselves signal arrival (a reader waits,
 * bounded by qcc_exchange_set_wait_limit, default 2 s, until none is the
 * empty mark, then marks them empty again), so there is no fence or flag
 * round trip.  A wait that runs out sets QCC_DEV_TIMEOUT in the workspace
 * status and leaves those columns of y unwritten; every rank must then
 * re-initialise its buffer (qcc_exchange_init) before the next call.  Replaces the NCCL all-reduce plus fp32 cast that
 * follow a sharded partial; the reference has no distributed path
 * (integration/freetoken_qcc/low_vram/adapter.py:106-107 refuses TP != 1).
 */
QCC_API int qcc_indexed_ffn_decode_allreduce(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                             int64_t n_records, int dtype, const void* ids, int ids_dtype, int n_ids,
                                             const int32_t* n_ids_dev, const uint8_t* token_mask, void* workspace,
                                             size_t workspace_bytes, void* y_out, int64_t ldy, int y_dtype,
                                             const float* y_in, int64_t ld_in, int64_t id_begin, int64_t id_end,
                                             void* const* exchange, size_t exchange_bytes, int world, int rank,
                                             cudaStream_t stream);

/* fp32 L2 norms of the cols columns of a row-major [rows, cols] matrix (row
 * stride ld elements, bf16 / fp16 / fp32), one pass with fp64 accumulation:
 * the down-column norms ||D[:, j]||_2 that weight the oracle's importance
 * (end_to_end/oracle_sparse_mlp.py:10-32 computes them in fp32 column chunks). */
QCC_API int qcc_column_norms(const void* w, int64_t ld, int64_t rows, int64_t cols, int dtype, float* out,
                             cudaStream_t stream);

/* Elementwise cast of n fp32 values to dtype (used after a cross-rank sum). */
QCC_API int qcc_cast_f32(const float* src, void* dst, int64_t n, int dtype, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Fused score producer + top-K (the runtime selector).
 *
 * Replaces runtime/cuda_selector.py:30-40 (latent_kernel + head_kernel, then
 * torch.topk(scores, k, sorted=False)) and the scoring of
 * runtime/selector.py:15-38 with one cooperative launch.  For each row b of x
 * [batch, hidden] (row stride ldx, elements):
 *   kind 0, ResidualFactorizedPredictor (predictor/models.py:17-36):
 *     r = silu(enc_w x + enc_b); u = silu(fc1_w r + fc1_b);
 *     v = fc2_w u + fc2_b + r;  z = LayerNorm(v; ln_eps) * ln_w + ln_b
 *   kind 1, FactorizedPredictor (predictor/models.py:6-14): z = enc_w x + enc_b
 *   scores = out_w z + out_b;
 *   ids[b * ld_ids + 0..k-1] = the k largest scores, ascending, ties to the
 *   lower index (the rule of qcc_select_topk).
 * Weights are nn.Linear layouts ([out, in], row-major), all in dtype, like x;
 * enc_w [latent, hidden] with the input normalisation folded in (enc_b =
 * -(enc_w) mean after dividing by std, runtime/selector.py:33-35); fc1_w,
 * fc2_w [latent, latent]; out_w [n_out, latent].  Every bias and ln_w / ln_b
 * may be NULL (zero / one).  Arithmetic is fp32.  scores, when not NULL,
 * receives the fp32 scores [batch, ld_scores].  latent <= 256.
 * The workspace (qcc_selector_workspace_bytes, zeroed once with
 * qcc_workspace_init) is left zeroed by every call; its status word is at
 * offset 0 (QCC_DEV_TIMEOUT: re-initialise it).  Rows beyond 32 run as
 * further launches on the same stream.
 * ------------------------------------------------------------------------- */
QCC_API size_t qcc_selector_workspace_bytes(int batch, int hidden, int latent, int n_out);

QCC_API int qcc_selector_scores_topk(const void* x, int64_t ldx, int batch, int hidden, int latent, int n_out,
                                     int kind, int dtype, const void* enc_w, const void* enc_b, const void* fc1_w,
                                     const void* fc1_b, const void* fc2_w, const void* fc2_b, const void* ln_w,
                                     const void* ln_b, float ln_eps, const void* out_w, const void* out_b, int k,
                                     int32_t* ids, int64_t ld_ids, float* scores, int64_t ld_scores,
                                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Block-sparse prefill.
 *
 * Replaces, for a prefill of n_tokens rows, the per-tile loop of
 * runtime/ffn.py:20-39 (TorchDynamicSparseFFN on each tile's ids) over ids that
 * come in whole blocks: block b stands for records [64b, 64b + 64), the
 * expansion of clustering/block_layout.py:61-64 and the block top-K of
 * oracle/importance.py:26-35.  Tokens form tiles of 128 rows (the last tile may
 * be partial); tile t uses the blocks tile_blocks[tile_offsets[t] ..
 * tile_offsets[t+1]), device arrays, each block at most once per tile, any
 * order.  For every row r of tile t:
 *   y[r] = sum over records n of t's blocks of silu(g_n . x_r) (u_n . x_r) d_n,
 * fp32 accumulation on the tensor cores; for bf16 / fp16 records the
 * activation is rounded to the weight type between the two products (as the
 * reference's CUDA path rounds it to fp16, runtime/cuda_indexed.py:28-30).
 * fp32 records run on kind::tf32: each product uses the tf32 part of its fp32
 * operands (x, the rows, the fp32 activation), the sums stay fp32.
 * ------------------------------------------------------------------------- */

/* Workspace for qcc_indexed_ffn_prefill on the current device (0 on bad
 * arguments).  Zero it once (qcc_workspace_init); calls leave it reusable. */
QCC_API size_t qcc_prefill_workspace_bytes(int64_t n_records, int hidden);

/* Byte offset of the int32 status word (QCC_DEV_* bits) in that workspace. */
QCC_API size_t qcc_prefill_workspace_status_offset(void);

/* x: [n_tokens, hidden] with row stride ldx (elements; ldx times the element
 * size a multiple of 16), in the records' dtype (bf16, fp16 or fp32); packed:
 * n_records records as packed by qcc_pack_records; tile_offsets:
 * ceil(n_tokens / 128) + 1 entries; y: [n_tokens, hidden], row stride ldy,
 * y_dtype.  Block ids out of range are skipped and set QCC_DEV_ID_RANGE in the
 * workspace status. */
QCC_API int qcc_indexed_ffn_prefill(const void* x, int64_t ldx, int n_tokens, int hidden, const void* packed,
                                    int64_t n_records, int dtype, const int32_t* tile_blocks,
                                    const int32_t* tile_offsets, void* workspace, size_t workspace_bytes, void* y,
                                    int64_t ldy, int y_dtype, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QCC_B200_H */
