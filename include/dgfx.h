/*
 * dgfx.h — C ABI of the B200 (sm_100a) implementation of DGF's in-memory
 * k-hop temporal neighbour sampler and of the sparse neighbour aggregation
 * that feeds its GNN layers.
 *
 * Conventions
 *   - Plain pointers and sizes only. Pointers named d_* are device pointers
 *     on the current CUDA device; everything else is host memory.
 *   - Every entry point returns a dgfx status (0 = DGFX_OK). On failure,
 *     dgfx_last_error() returns the message (per host thread). Status codes
 *     reuse absl's numbering so a binding can map INVALID_ARGUMENT and
 *     FAILED_PRECONDITION to Python ValueError exactly like the reference's
 *     status caster (dgf/src/util/status_caster.h:17-21, 83-88).
 *   - Work is enqueued on the caller's stream. Temporaries live in a
 *     caller-provided workspace whose size the matching *_workspace_size
 *     query returns; the library allocates no per-call device memory.
 *   - No entry point falls back to a CPU implementation.
 */
#ifndef DGFX_H_
#define DGFX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct CUstream_st* dgfx_stream; /* == cudaStream_t */

enum {
  DGFX_OK = 0,
  DGFX_ERR_INVALID_ARGUMENT = 3,
  DGFX_ERR_NOT_FOUND = 5,
  DGFX_ERR_FAILED_PRECONDITION = 9,
  DGFX_ERR_INTERNAL = 13,
  DGFX_ERR_CUDA = 100,
  DGFX_ERR_WORKSPACE = 101,
  DGFX_ERR_UNSUPPORTED = 102
};

enum { DGFX_F32 = 0, DGFX_BF16 = 1 };

/* Sampling modes. RANDOM and FIRST are the reference's two modes
 * (create_sampler(debug_sampling=False/True), in_memory_sampler.py:349-363,
 * applied in SampleBuilder::RecursiveGrow, in_memory_sampler_ext.cc:250-279).
 * MOST_RECENT has no reference counterpart: the newest k edges whose
 * timestamp is <= the seed timestamp; non-temporal edgesets sample as RANDOM. */
enum { DGFX_MODE_RANDOM = 0, DGFX_MODE_FIRST = 1, DGFX_MODE_MOST_RECENT = 2 };

/* Message of the last failure on this host thread ("" if none). */
const char* dgfx_last_error(void);
/* Library ABI version (major * 100 + minor). */
int dgfx_version(void);

/* ------------------------------------------------------------------------
 * Adjacency index (CSR of one direction of one edgeset).
 * Replaces AdjacencyIndex::CreateFromEdgeList (in_memory_sampler.cc:220-257)
 * behind BuildAdjacencyIndex (in_memory_sampler_ext.cc:1020-1093): ids are
 * validated (first invalid edge reported with the reference's message), the
 * edges are sorted by (source, timestamp, target) with duplicates kept, and
 * the row pointers are filled. Layout: rowptr int64[num_src + 1], col
 * int32[E], ts int64[E] (temporal only), edge_pos int64[E] where
 * edge_pos[e] = CSR position of original edge e (only when masking is
 * configured; the inverse of the reference's parallel edge_idxs array).
 * num_src / num_dst are the edgeset's source / target node counts *before*
 * the reversal, as in the reference. Synchronises `stream` once to report
 * invalid ids.
 * ------------------------------------------------------------------------ */
int dgfx_csr_build_workspace_size(int64_t num_edges, int64_t num_src,
                                  int64_t num_dst, int has_ts, size_t* bytes);
int dgfx_csr_build(const int64_t* d_src, const int64_t* d_dst,
                   const int64_t* d_ts, int64_t num_edges, int64_t num_src,
                   int64_t num_dst, int reversed, int64_t* d_rowptr,
                   int32_t* d_col, int64_t* d_ts_out, int64_t* d_edge_pos,
                   void* d_workspace, size_t workspace_bytes,
                   dgfx_stream stream);

/* Device view of one built index. rowptr == NULL marks "not built". */
typedef struct dgfx_csr_view {
  const int64_t* rowptr;
  const int32_t* col;
  const int64_t* ts;       /* NULL: non-temporal edgeset */
  const int64_t* edge_pos; /* NULL: no masking on this edgeset */
  int64_t num_src;
  int64_t num_dst;
  int64_t num_edges;
} dgfx_csr_view;

/* ------------------------------------------------------------------------
 * Sampler. Replaces the native Sampler of _in_memory_sampler_ext
 * (CreateSampler in_memory_sampler_ext.cc:1216-1246; Sampler::Sample
 * :418-533 with SampleBuilder::Grow/RecursiveGrow :231-370).
 *
 * Plan: node i (node 0 = root) has nodeset node_nodeset[i] and plan edges
 * [node_first_edge[i], node_first_edge[i] + node_num_edges[i]); plan edge j
 * walks edgeset edge_edgeset[j] (edge_reversed[j]: backward index) taking up
 * to edge_hop_width[j] neighbours into plan node edge_child[j]. Mirrors
 * SamplingPlan (in_memory_sampler.h:172-239).
 * forward[e] / backward[e]: the indices of edgeset e (rowptr NULL if the plan
 * does not walk that direction). Views are borrowed: they must outlive the
 * sampler. Output per seed matches the reference: nodes relabelled in
 * first-discovery depth-first order (all occurrences when with_replacement),
 * edges deduplicated and sorted by (src_local, dst_local) per edgeset.
 * ------------------------------------------------------------------------ */
typedef struct dgfx_sampler dgfx_sampler;

int dgfx_sampler_create(int32_t num_plan_nodes, const int32_t* node_nodeset,
                        const int32_t* node_first_edge,
                        const int32_t* node_num_edges, int32_t num_plan_edges,
                        const int32_t* edge_edgeset,
                        const int32_t* edge_reversed,
                        const int32_t* edge_hop_width,
                        const int32_t* edge_child, int32_t with_replacement,
                        int32_t num_nodesets, const int64_t* num_nodes,
                        int32_t num_edgesets, const dgfx_csr_view* forward,
                        const dgfx_csr_view* backward, int32_t mode,
                        int32_t edgeset_to_mask, uint64_t seed,
                        dgfx_sampler** out);
void dgfx_sampler_destroy(dgfx_sampler* sampler);

/* Kernel choice of dgfx_sampler_sample (no counterpart in the reference,
 * whose sampler is host code). kind 0 (default): the warp sampler (one warp
 * per seed over the occupied tree positions, in shared memory, 32 to 128
 * entries by the plan's tree size) when the plan allows it; seeds whose
 * trees outgrow it are redone by the large-tree tier (one CTA of four warps
 * per seed, up to 512 entries), and seeds beyond that by the padded sampler
 * (one CTA per seed over all tree positions). kind 1: the padded sampler
 * for every seed. kind 2: the warp sampler with the padded sampler behind
 * it (no large-tree tier). All give identical batches in every mode (same
 * random stream). dgfx_sampler_kernel_info reports the warp sampler's and
 * the large-tree tier's per-seed entry capacities under the current kind
 * (0 when not used; large_capacity may be NULL). */
int dgfx_sampler_set_kernel(dgfx_sampler* sampler, int32_t kind);
int dgfx_sampler_kernel_info(const dgfx_sampler* sampler, int32_t* warp_capacity,
                             int32_t* large_capacity);
/* Of the last dgfx_sampler_sample's seeds (synchronises `stream`):
 * out2[0] = seeds a warp tier finished, out2[1] = seeds whose trees
 * outgrew every warp tier and were finished by the padded sampler. */
int dgfx_sampler_kernel_stats(dgfx_sampler* sampler, dgfx_stream stream, int64_t* out2);

/* Positions of the padded per-seed expansion tree (an upper bound on the
 * nodes of one sample). */
int dgfx_sampler_tree_size(const dgfx_sampler* sampler, int64_t* positions);
int dgfx_sampler_workspace_size(const dgfx_sampler* sampler, int64_t num_seeds,
                                size_t* bytes);
int dgfx_sampler_output_capacity(const dgfx_sampler* sampler,
                                 int64_t num_seeds, int64_t* max_nodes,
                                 int64_t* max_edges);

/* Merged batch written by dgfx_sampler_sample (all device pointers).
 *   node_ids[node_offsets[s*B + i] .. node_offsets[s*B + i + 1]) are the
 *     "#idx" of nodeset s in sample i, in local-id order (nodeset-major, then
 *     sample); node_offsets has num_nodesets*B + 1 entries.
 *   edge_src / edge_dst[edge_offsets[e*B + i] .. edge_offsets[e*B + i + 1])
 *     are the local-id adjacency rows of edgeset e in sample i
 *     (EdgesToNumpyArray layout, in_memory_sampler_nb.h:31-57).
 * Capacities come from dgfx_sampler_output_capacity. */
typedef struct dgfx_sample_out {
  int64_t* node_ids;
  int64_t* node_offsets;
  int64_t* edge_src;
  int64_t* edge_dst;
  int64_t* edge_offsets;
} dgfx_sample_out;

/* Samples one subgraph per seed. d_seed_ts (int64[B]) enables the temporal
 * cutoff (edge ts <= seed ts); d_masked_edges (int64[B], -1 = none) masks one
 * edge of the masked edgeset per seed. call_index selects the random stream
 * (Philox4x32-10 keyed by the sampler seed; counter = (call, seed slot, tree
 * position, plan edge)); call_index == DGFX_CALL_INDEX_DEVICE takes it from
 * a counter in device memory that each call advances, so a call captured in
 * a CUDA graph draws a new stream on every replay (the call issues only
 * kernels and memsets; no host synchronisation). Asynchronous: device-side
 * failures (seed out of range, timestamps missing for a temporal index) are
 * latched and reported by dgfx_sampler_check. */
#define DGFX_CALL_INDEX_DEVICE (~0ull)
int dgfx_sampler_sample(dgfx_sampler* sampler, const int64_t* d_seeds,
                        const int64_t* d_seed_ts, const int64_t* d_masked_edges,
                        int64_t num_seeds, uint64_t call_index,
                        const dgfx_sample_out* out, void* d_workspace,
                        size_t workspace_bytes, dgfx_stream stream);

/* Same as dgfx_sampler_sample but allocates nothing and takes no workspace:
 * for callers that cannot allocate device memory when they sample (a
 * framework that owns the device's memory pool, a fixed-arena serving
 * runtime, a plugin called where allocation is not allowed). Its scratch is
 * one file-scope 64 MiB device array of this library, held on every GPU that
 * loads the library until exit; a call whose dgfx_sampler_workspace_size
 * exceeds 64 MiB fails with DGFX_ERR_INVALID_ARGUMENT. The array's address
 * is looked up on the first call on each device (make that call before any
 * stream capture) and kept for the life of the process: a device reset
 * invalidates it, so do not call this entry point again after
 * cudaDeviceReset in the same process. Calls share the array: calls that
 * overlap on the GPU race. This entry point has no counterpart in the
 * reference. */
int dgfx_sampler_sample_noalloc(dgfx_sampler* sampler, const int64_t* d_seeds,
                                const int64_t* d_seed_ts,
                                const int64_t* d_masked_edges,
                                int64_t num_seeds, uint64_t call_index,
                                const dgfx_sample_out* out, dgfx_stream stream);

/* Same result as dgfx_sampler_sample, split over two streams so that
 * back-to-back batches overlap: the first sampling kernel runs on `stream`;
 * the kernel that finishes the seeds with large sampled trees, the offset
 * scans and the compaction of `out` run on `tail_stream` after it. `out` is
 * complete in `tail_stream` order; `stream` is free for the next batch as
 * soon as the first kernel ends. The next call on the same sampler waits on
 * its `stream` for this call's tail before it touches the workspace, so
 * callers that want two batches in flight alternate two samplers (and two
 * workspaces). dgfx_sampler_check / _stats / _kernel_stats also wait for the
 * tail. `tail_stream` must differ from `stream`. Identical batches to
 * dgfx_sampler_sample for the same call_index. No reference counterpart. */
int dgfx_sampler_sample_split(dgfx_sampler* sampler, const int64_t* d_seeds,
                              const int64_t* d_seed_ts,
                              const int64_t* d_masked_edges,
                              int64_t num_seeds, uint64_t call_index,
                              const dgfx_sample_out* out, void* d_workspace,
                              size_t workspace_bytes, dgfx_stream stream,
                              dgfx_stream tail_stream);

/* Synchronises `stream` and reports the latched status of the last
 * dgfx_sampler_sample (reference messages, e.g. "The source node idx 7 is out
 * of bounds. Should be lower than 4"). */
int dgfx_sampler_check(dgfx_sampler* sampler, dgfx_stream stream);

/* Work counters of the last dgfx_sampler_sample (synchronises `stream`):
 * out3[0] = adjacency rows expanded, out3[1] = neighbours sampled,
 * out3[2] = timestamp binary-search probes. They feed the algorithmic-byte
 * count of the sampler's roofline. No reference counterpart. */
int dgfx_sampler_stats(dgfx_sampler* sampler, dgfx_stream stream,
                       int64_t* out3);

/* ------------------------------------------------------------------------
 * Feature gather: out[i, :] = table[row_ids[i], :] for row_bytes-wide rows
 * (row_bytes a multiple of 16). Replaces add_features_to_samples'
 * full_feature_value[node_idxs] (in_memory_sampler.py:313-346).
 * Ids outside [0, num_table_rows) produce zero rows.
 * ------------------------------------------------------------------------ */
int dgfx_gather_rows(const void* d_table, int64_t num_table_rows,
                     int64_t row_bytes, const int64_t* d_row_ids,
                     int64_t num_rows, void* d_out, dgfx_stream stream);

/* Same, for the rows [*d_begin, *d_end) of d_row_ids with both bounds read
 * on the device (at most max_rows rows; out row i <- d_row_ids[*d_begin + i]).
 * Lets a node set of a merged batch be gathered straight from the batch's
 * offsets, without a host synchronisation. */
int dgfx_gather_rows_ranged(const void* d_table, int64_t num_table_rows,
                            int64_t row_bytes, const int64_t* d_row_ids,
                            const int64_t* d_begin, const int64_t* d_end,
                            int64_t max_rows, void* d_out, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Aggregation.
 * dgfx_spmm_csr: Y[r, :] = scale_r * sum_j val[j] * X[col[j], :] over row r
 * of a CSR matrix (rows = message targets, cols = message sources), the
 * sparse_deferred `SparseMatrix @ dense` form (homo_gnn_sparse_deferred.py:
 * 138-161, message_passing.py:24-38). val == NULL means 1. normalize = 1
 * gives the mean pooling of hetero_gnn.py:283-295: scale_r =
 * 1 / max(deg_r, 1). X and Y are row-major [*, feat]; fp32 accumulation.
 * Deterministic (fixed summation order).
 * ------------------------------------------------------------------------ */
int dgfx_spmm_workspace_size(int64_t num_rows, int64_t nnz, int64_t feat,
                             size_t* bytes);
int dgfx_spmm_csr(const int64_t* d_rowptr, const int32_t* d_col,
                  const float* d_val, int64_t num_rows, int64_t num_cols,
                  int64_t nnz, const void* d_x, int x_dtype, void* d_y,
                  int y_dtype, int64_t feat, int32_t normalize,
                  void* d_workspace, size_t workspace_bytes,
                  dgfx_stream stream);

/* jax.ops.segment_sum(data, segment_ids, num_segments) as called at
 * hetero_gnn.py:283-287; mean = 1 adds the division by max(count, 1) of
 * hetero_gnn.py:288-295. Ids outside [0, num_segments) are dropped (jax
 * semantics). indices_are_sorted = 1 selects a deterministic segmented
 * reduction; otherwise fp32 atomic accumulation is used. */
int dgfx_segment_sum_workspace_size(int64_t num_items, int64_t feat,
                                    int64_t num_segments, size_t* bytes);
int dgfx_segment_sum(const void* d_data, int data_dtype,
                     const int64_t* d_segment_ids, int64_t num_items,
                     int64_t feat, int64_t num_segments, int32_t mean,
                     int32_t indices_are_sorted, void* d_out, int out_dtype,
                     void* d_workspace, size_t workspace_bytes,
                     dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Segment softmax aggregation (graph attention). Replaces the relation
 * attention of dgf/src/learning/jax/layers/hetero_graph_attention_network.py:
 * 242-263 (segment_max, exp, segment_sum, divide, weighted segment_sum):
 *   d_out[t, h, :] = sum_{e: id(e) = t} w[e, h] * msg[e, h, :]
 *   w[e, h] = exp(l[e, h] - m[t, h]) / (sum_{e'} exp(l[e', h] - m[t, h]) + 1e-9)
 *   m[t, h] = max_{e: id(e) = t} l[e, h]
 * d_logits fp32 [n, heads]; d_messages [n, heads, head_dim] (msg_dtype;
 * head_dim a multiple of 4 for fp32, 8 for bf16; heads * head_dim * element
 * size <= 2 KB); d_ids int64 [n] (ids outside [0, nseg) are dropped;
 * sorted != 0 promises ascending ids); d_out [nseg, heads, head_dim]
 * (out_dtype), zero rows for empty segments. Segments are split into
 * chunks of 256 items (one warp each); chunk states merge in chunk order, so
 * results are deterministic. With sorted ids, heads dividing 32 and rows of
 * at most 32 16-byte slices, a chunk's per-head maximum is taken from its
 * contiguous logits first and warps of a persistent grid take chunks from a
 * counter; otherwise a running (online) softmax over the chunk. Segments
 * whose logits are all -inf give zero rows.
 * ------------------------------------------------------------------------ */
int dgfx_segment_softmax_workspace_size(int64_t num_items, int64_t num_segments,
                                        int32_t heads, int64_t head_dim,
                                        int msg_dtype, int32_t sorted,
                                        size_t* bytes);
int dgfx_segment_softmax(const float* d_logits, int32_t heads,
                         const void* d_messages, int msg_dtype, int64_t head_dim,
                         const int64_t* d_ids, int64_t n, int64_t nseg,
                         int32_t sorted, void* d_out, int out_dtype,
                         void* d_workspace, size_t workspace_bytes,
                         dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Dense layer after aggregation on the tensor cores (tcgen05, sm_100a).
 * Replaces the nn.Dense (+ activation) that follows the neighbour
 * aggregation (dgf/src/learning/jax/layers/hetero_gnn.py:302-312,
 * standard.py:238-270): d_y[m, n] = act(concat[d_x1, d_x2] @ d_w^T + d_bias)
 * with d_x1 bf16 [m, k1], d_x2 bf16 [m, k2] (NULL when k2 = 0), d_w bf16
 * [n, k1 + k2] (output-major, torch Linear layout), d_bias fp32 [n] or NULL,
 * act = ReLU when relu != 0 else identity; fp32 accumulation, bf16 output
 * (round to nearest). k1 >= 64; k1, k2 and n multiples of 64; all operands
 * 16-byte aligned. A pipeline wait that runs out (2 s) is latched and
 * reported by dgfx_dense_check (synchronises the stream) as
 * DGFX_ERR_INTERNAL.
 * ------------------------------------------------------------------------ */
int dgfx_dense_concat_bf16(const void* d_x1, int64_t k1, const void* d_x2,
                           int64_t k2, int64_t m, const void* d_w,
                           const float* d_bias, int64_t n, int32_t relu,
                           void* d_y, dgfx_stream stream);
int dgfx_dense_check(dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Halo feature exchange (node-range-partitioned features across ranks).
 * Replaces the Beam CoGroupByKey feature join of
 * dgf/src/sampling/beam_semi_distributed_sampler_v2.py:271-387; the rows
 * themselves move in one NCCL all-to-all issued by the host driver.
 * dgfx_halo_partition: stable sort of requested ids by owner
 * (owner = id / rows_per_rank, clamped to [0, world)); d_sorted_ids[j] =
 * d_ids[d_perm[j]]; d_counts[w] = ids owned by rank w.
 * dgfx_gather_rows_local: out[i] = table[ids[i] - id_base] (zero row if
 * outside [0, local_rows)).
 * dgfx_scatter_rows: out[perm[i]] = rows[i].
 * ------------------------------------------------------------------------ */
int dgfx_halo_partition_workspace_size(int64_t n, int32_t world, size_t* bytes);
int dgfx_halo_partition(const int64_t* d_ids, int64_t n, int64_t rows_per_rank,
                        int32_t world, int64_t* d_sorted_ids, uint32_t* d_perm,
                        int64_t* d_counts, void* d_workspace,
                        size_t workspace_bytes, dgfx_stream stream);
int dgfx_gather_rows_local(const void* d_table, int64_t local_rows,
                           int64_t row_bytes, const int64_t* d_ids, int64_t n,
                           int64_t id_base, void* d_out, dgfx_stream stream);
int dgfx_scatter_rows(const void* d_rows, int64_t n, int64_t row_bytes,
                      const uint32_t* d_perm, void* d_out, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Peer-memory feature gather (one kernel instead of the all-to-all halo
 * exchange when the ranks' GPUs have peer access, e.g. over NVSwitch).
 * Each rank allocates its feature partition with dgfx_device_alloc, shares
 * it with dgfx_ipc_get_handle (64-byte CUDA IPC handle) and opens the other
 * ranks' handles with dgfx_ipc_open; d_tables is a device array of the
 * `world` partition pointers (its own included). dgfx_gather_rows_p2p:
 * out[i] = partition(o)[id - o * rows_per_rank] for id = d_row_ids[*d_begin
 * + i], o = id / rows_per_rank (zero row for ids outside [0, num_nodes)),
 * at most max_rows rows, bounds read on the device. Remote rows are read
 * with plain loads over NVLink (no TMA, no multicast).
 * ------------------------------------------------------------------------ */
int dgfx_device_alloc(size_t bytes, void** d_ptr);
int dgfx_device_free(void* d_ptr);
int dgfx_ipc_get_handle(const void* d_ptr, void* handle64);
int dgfx_ipc_open(const void* handle64, void** d_ptr);
int dgfx_ipc_close(void* d_ptr);
int dgfx_gather_rows_p2p(const void* const* d_tables, int32_t world,
                         int64_t rows_per_rank, int64_t num_nodes,
                         int64_t row_bytes, const int64_t* d_row_ids,
                         const int64_t* d_begin, const int64_t* d_end,
                         int64_t max_rows, void* d_out, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Bulk peer exchange of feature rows (same result as dgfx_gather_rows_p2p;
 * every byte that crosses NVLink moves in contiguous runs, every random row
 * access is to this GPU's own HBM). Each rank owns one exchange buffer of
 * dgfx_exchange_buffer_size bytes (dgfx_device_alloc, shared by CUDA IPC like
 * the partitions, zeroed once): per-owner request counts, per-owner request-id
 * slots of slot_rows ids, barrier flags and per-owner row inboxes of slot_rows
 * rows. A step is three stream-ordered launches separated by group barriers
 * (dgfx_exchange_barrier, or any group-wide barrier on the same stream):
 *   dgfx_exchange_partition (requester): zeroes this rank's counts and puts
 *     ids[*d_begin + i] (i < min(*d_end - *d_begin, max_rows)) into the slot
 *     of its owner o = id / rows_per_rank; d_req_pos[o * slot_rows + k] = i.
 *     Ids outside [0, num_nodes) get a zero row in d_out here.
 *   -- barrier --
 *   dgfx_exchange_serve (owner): reads every requester's slot for this rank
 *     (contiguous peer reads), gathers the rows from the local partition and
 *     writes them into that requester's inbox (contiguous peer stores); its
 *     own requests go straight to d_out.
 *   -- barrier --
 *   dgfx_exchange_scatter (requester): d_out[d_req_pos[...]] = inbox rows.
 * dgfx_exchange_barrier: every rank publishes `epoch` (increasing per call,
 * same sequence on all ranks, starting at 1) in the other ranks' flags and
 * waits for theirs, at most max_wait_ns; a wait that runs out sets the
 * timeout flag instead of hanging. With epoch 0 the kernel takes the next
 * epoch from a counter in this rank's exchange buffer, so the launches can
 * be captured in a CUDA graph and replayed (every rank must then use epoch
 * 0 for all its barriers, in the same sequence).
 * Local replica (optional): d_hot_slot int32[num_nodes] maps a node to its
 * row in this rank's d_replica table (a read-only copy of frequently
 * requested rows, replica_rows x row_bytes), -1 elsewhere. Requests for such
 * nodes never cross NVLink: the partition puts them in an extra slot and the
 * serve launch copies their rows locally. NULL / 0 disables it.
 * dgfx_exchange_check (synchronises the stream) reports and clears the flags:
 * slot overflow (a slot needed more than slot_rows ids; rows were dropped) as
 * DGFX_ERR_WORKSPACE, barrier timeout as DGFX_ERR_FAILED_PRECONDITION.
 * d_exchanges is a device array of the `world` exchange-buffer pointers (own
 * included); d_req_pos holds (world + 1) * slot_rows int32 and stays on this
 * rank.
 * world <= 16.
 * ------------------------------------------------------------------------ */
int dgfx_exchange_buffer_size(int32_t world, int64_t slot_rows,
                              int64_t row_bytes, size_t* bytes);
int dgfx_exchange_partition(void* d_exchange, int32_t world, int64_t slot_rows,
                            int64_t rows_per_rank, int64_t num_nodes,
                            int64_t row_bytes, const int64_t* d_row_ids,
                            const int64_t* d_begin, const int64_t* d_end,
                            int64_t max_rows, const int32_t* d_hot_slot,
                            int32_t* d_req_pos, void* d_out,
                            dgfx_stream stream);
int dgfx_exchange_serve(const void* const* d_exchanges, int32_t world,
                        int32_t rank, int64_t slot_rows, int64_t rows_per_rank,
                        int64_t row_bytes, const void* d_table,
                        int64_t local_rows, const void* d_replica,
                        int64_t replica_rows, const int32_t* d_req_pos,
                        void* d_out, dgfx_stream stream);
int dgfx_exchange_scatter(const void* const* d_exchanges, int32_t world,
                          int32_t rank, int64_t slot_rows, int64_t row_bytes,
                          const int32_t* d_req_pos, void* d_out,
                          dgfx_stream stream);
int dgfx_exchange_barrier(const void* const* d_exchanges, int32_t world,
                          int32_t rank, uint32_t epoch, uint64_t max_wait_ns,
                          dgfx_stream stream);
int dgfx_exchange_check(const void* d_exchange, int32_t world,
                        dgfx_stream stream);
/* The whole exchange of one gather in one call: partition, barrier with
 * `epoch`, serve, barrier with the next epoch (epoch + 1, wrapping to 1
 * after 2^31 - 1), scatter; the same launches as the five calls above, with
 * no host code between them. The caller advances its epoch by two; with
 * epoch 0 both barriers take their epochs on the device (see
 * dgfx_exchange_barrier). No reference counterpart. */
int dgfx_exchange_gather(const void* const* d_exchanges, void* d_exchange,
                         int32_t world, int32_t rank, int64_t slot_rows,
                         int64_t rows_per_rank, int64_t num_nodes,
                         int64_t row_bytes, const int64_t* d_row_ids,
                         const int64_t* d_begin, const int64_t* d_end,
                         int64_t max_rows, const int32_t* d_hot_slot,
                         int32_t* d_req_pos, const void* d_table,
                         int64_t local_rows, const void* d_replica,
                         int64_t replica_rows, void* d_out, uint32_t epoch,
                         uint64_t max_wait_ns, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Edge creation times from node creation times. Replaces the numpy body of
 * propagate_timestamp_to_edges (dgf/src/transform/temporal.py:95-103):
 * d_out[e] = max(d_src_ts[d_src[e]], d_dst_ts[d_dst[e]]); with one of the
 * two node timestamp arrays NULL, the other endpoint's time. Endpoint ids are
 * bounds-checked against num_src / num_dst; the first edge with an
 * out-of-range id is reported as DGFX_ERR_INVALID_ARGUMENT. d_workspace:
 * 8 bytes. Synchronises `stream` once.
 * ------------------------------------------------------------------------ */
int dgfx_edge_timestamps(const int64_t* d_src_ts, int64_t num_src,
                         const int64_t* d_dst_ts, int64_t num_dst,
                         const int64_t* d_src, const int64_t* d_dst,
                         int64_t num_edges, int64_t* d_out, void* d_workspace,
                         dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Random-walk negative sampling. Replaces Sampler::RandomWalkNegativeSampling
 * with RandomWalkNegativeSamplerHelper (dgf/src/sampling/
 * in_memory_sampler_ext.cc:774-948): per seed, num_walks walks down the
 * sampler's plan (uniform plan edge, uniform neighbour, stop at a node
 * without neighbours); visits of nodes of the target edge set's target node
 * set are counted (not the seed itself on a homogeneous edge set); nodes the
 * seed links to in the target edge set's forward index are dropped; the
 * num_negatives_per_seed most visited (ties: smaller id first) fill the row
 * of d_out (int64 [num_seeds, num_negatives_per_seed]), the rest are uniform
 * draws over the target node set (never the seed of a homogeneous edge set).
 * Draws come from Philox4x32-10 keyed by the sampler seed; call_index selects
 * the stream. Errors: "Invalid target_edgeset_idx"; no forward index for the
 * edge set; a target node set with no node to draw for the fallback slots.
 * Asynchronous: seeds outside the root node set, a full visit table and
 * exhausted fallback draws are latched in the workspace and reported by
 * dgfx_random_walk_negatives_check (which synchronises `stream`).
 * ------------------------------------------------------------------------ */
int dgfx_random_walk_negatives_workspace_size(const dgfx_sampler* sampler,
                                              int64_t num_seeds,
                                              int32_t target_edgeset,
                                              int32_t num_walks,
                                              int32_t num_negatives_per_seed,
                                              size_t* bytes);
int dgfx_random_walk_negatives(dgfx_sampler* sampler, const int64_t* d_seeds,
                               int64_t num_seeds, int32_t target_edgeset,
                               int32_t num_walks, int32_t num_negatives_per_seed,
                               uint64_t call_index, int64_t* d_out,
                               void* d_workspace, size_t workspace_bytes,
                               dgfx_stream stream);
int dgfx_random_walk_negatives_check(const void* d_workspace, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Raw node id -> node index. Replaces ByteIdToIdxMapper / PairMapping
 * (dgf/src/io/io_ext.cc:26-170) and the integer-id dictionary of
 * _read_node_set (dgf/src/io/graph_in_memory.py:80-125) used when a GF graph
 * is loaded. Ids are read in place on the device:
 *   DGFX_IDS_INT64  d_ids = int64[num_ids]
 *   DGFX_IDS_FIXED  d_ids = bytes, num_ids rows of `width` bytes (numpy 'S')
 *   DGFX_IDS_VAR    d_ids = bytes, d_offsets = int64[num_ids + 1] (Arrow binary)
 * A byte id is its bytes without trailing zero bytes; a repeated id maps to
 * its last position. The index borrows d_ids / d_offsets (keep them alive).
 * Lookup writes the index of every query id (-1 when absent) and, if
 * `mismatch` is non-null, synchronises and stores the largest position of an
 * absent id (-1 if none). Integer ids only match integer ids. Lookups on one
 * index are serialised by the caller.
 * ------------------------------------------------------------------------ */
enum { DGFX_IDS_INT64 = 0, DGFX_IDS_FIXED = 1, DGFX_IDS_VAR = 2 };
typedef struct dgfx_id_index dgfx_id_index;
/* Table memory: d_table (8-byte aligned, dgfx_id_index_table_bytes) is
 * borrowed for the index's lifetime; with d_table NULL the index allocates
 * its own. Creation synchronises `stream`. */
int dgfx_id_index_table_bytes(int64_t num_ids, size_t* bytes);
int dgfx_id_index_create(int32_t kind, const void* d_ids, const int64_t* d_offsets,
                         int64_t width, int64_t num_ids, void* d_table,
                         size_t table_bytes, dgfx_stream stream, dgfx_id_index** out);
void dgfx_id_index_destroy(dgfx_id_index* index);
int dgfx_id_index_lookup(const dgfx_id_index* index, int32_t kind, const void* d_ids,
                         const int64_t* d_offsets, int64_t width, int64_t num_ids,
                         int64_t* d_out, int64_t* mismatch, dgfx_stream stream);

/* Keeps the pairs whose two indices are >= 0 (dangling-edge removal,
 * graph_in_memory.py:185-198), in order: d_out_src / d_out_dst get the kept
 * pairs, d_out_pos (nullable) their positions in the input; *num_kept is
 * read back (synchronises `stream`). */
int dgfx_compact_pairs_workspace_size(int64_t num_pairs, size_t* bytes);
int dgfx_compact_pairs(const int64_t* d_src, const int64_t* d_dst, int64_t num_pairs,
                       int64_t* d_out_src, int64_t* d_out_dst, int64_t* d_out_pos,
                       int64_t* num_kept, void* d_workspace, size_t workspace_bytes,
                       dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Causal windows of per-node time series. Replaces the per-node loop of
 * filter_timeseries_by_timestamp (dgf/src/sampling/temporal.py:24-130).
 * Node r's timestamp series is d_times[d_row_offsets[r] .. d_row_offsets[r+1])
 * (sorted). For query i (node d_rows[i], cutoff d_cutoffs[i]) the window is
 * the entries with time <= cutoff, keeping the last max_len of them
 * (max_len < 0: all): d_rel_start[i] = its first entry relative to the row,
 * d_len[i] = its length. d_workspace: 8 bytes. Synchronises `stream`; a row
 * id outside [0, num_rows) is DGFX_ERR_INVALID_ARGUMENT.
 * dgfx_gather_segments copies segment i, d_len[i] elements of elem_bytes
 * starting at element d_start[i] of d_values, to element d_out_offsets[i] of
 * d_out (packed ragged output).
 * ------------------------------------------------------------------------ */
int dgfx_timeseries_windows(const int64_t* d_row_offsets, const int64_t* d_times,
                            int64_t num_rows, const int64_t* d_rows,
                            const int64_t* d_cutoffs, int64_t n, int64_t max_len,
                            int64_t* d_rel_start, int64_t* d_len, void* d_workspace,
                            dgfx_stream stream);
int dgfx_gather_segments(const void* d_values, int64_t elem_bytes, const int64_t* d_start,
                         const int64_t* d_len, const int64_t* d_out_offsets, int64_t n,
                         void* d_out, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Subgraph around a set of seeds. Replaces the numbering and edge set of
 * SubGraphExtractor (dgf/src/sampling/in_memory_sampler_ext.cc:600-772) as
 * the union of a merged batch of per-seed samples (dgfx_sample_out layout,
 * one sample per seed): the seeds are the first `batch` nodes of
 * root_nodeset (ids in seed order; a repeated seed node maps to its last
 * seed id), every other node is numbered in its node set in order of its
 * first (seed index, local id) occurrence, and the edges, mapped to these
 * ids, are deduplicated and sorted by (source, target) per edge set.
 * edge_src_nodeset / edge_dst_nodeset (host, num_edgesets) give each edge
 * set's endpoint node sets. Outputs: d_out_node_ids (total_nodes capacity)
 * node-set major with out_node_counts (host, num_nodesets);
 * d_out_src / d_out_dst (total_edges capacity) edge-set major with
 * out_edge_counts (host). Synchronises the stream. total_nodes < 2^28.
 * ------------------------------------------------------------------------ */
int dgfx_subgraph_union_workspace_size(int64_t total_nodes, int64_t total_edges,
                                       size_t* bytes);
int dgfx_subgraph_union(const int64_t* d_node_ids, const int64_t* d_node_offsets,
                        const int64_t* d_edge_src, const int64_t* d_edge_dst,
                        const int64_t* d_edge_offsets, int64_t batch,
                        int32_t num_nodesets, int32_t num_edgesets,
                        int32_t root_nodeset, const int32_t* edge_src_nodeset,
                        const int32_t* edge_dst_nodeset, int64_t total_nodes,
                        int64_t total_edges, int64_t* d_out_node_ids,
                        int64_t* out_node_counts, int64_t* d_out_src,
                        int64_t* d_out_dst, int64_t* out_edge_counts,
                        void* d_workspace, size_t workspace_bytes,
                        dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Merged-batch adjacency with padding. Replaces the adjacency part of
 * merge_graphs (dgf/src/transform/merge.py:165-197) for a merged batch
 * (dgfx_sample_out layout: offsets set-major, then sample, trailing total):
 * d_out_src / d_out_dst[k] for the k-th edge of edge set `edgeset` over all
 * samples in order = its local ids plus the sample's first node in the
 * source / target node set (d_node_offsets[ns * batch + i] -
 * d_node_offsets[ns * batch]); entries from the real edge count up to
 * num_out are padding edges (sentinel_src, sentinel_dst); real edges past
 * num_out are dropped (the caller checks the counts first).
 * ------------------------------------------------------------------------ */
int dgfx_merge_edgeset(const int64_t* d_node_offsets,
                       const int64_t* d_edge_offsets, const int64_t* d_edge_src,
                       const int64_t* d_edge_dst, int64_t batch, int32_t edgeset,
                       int32_t src_nodeset, int32_t dst_nodeset,
                       int64_t num_out, int64_t sentinel_src,
                       int64_t sentinel_dst, int64_t* d_out_src,
                       int64_t* d_out_dst, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Sparse-matrix helpers around dgfx_spmm_csr.
 * dgfx_csr_add_diagonal: from the structure CSR of S = A + A^T (implicit
 * values 1; built by dgfx_csr_build over the concatenated edge list) writes
 * M = S + diag * I with one diagonal entry appended per row (out_rowptr
 * [n + 1], out_col / out_val [nnz + n]); normalize_symmetric != 0 scales
 * entry (r, c) by 1 / sqrt(d_r d_c), d = row sums of M. Replaces the
 * propagation matrices the reference builds with sparse_deferred:
 * GCN (adj + adj.T).add_eye().normalize_symmetric()
 * (dgf/src/learning/jax/layers/homo_gnn_sparse_deferred.py:293) and GIN
 * (adj + adj.T).add_eye(1 + eps) (:526).
 * dgfx_csr_row_ids: out[j] = row of CSR entry j (to transpose a CSR for the
 * SpMM's backward pass: rows of the transpose = columns of the matrix).
 * dgfx_segment_counts: counts[s] = items with id s (ids outside [0, n_seg)
 * are skipped), the degrees of jax.ops.segment_sum's mean pooling
 * (dgf/src/learning/jax/layers/hetero_gnn.py:288-293).
 * dgfx_gather_rows_scaled: out[i, :] = src[ids[i], :] (/ max(counts[ids[i]],
 * 1) if counts != NULL), zero rows for ids outside [0, num_segments): the
 * gradient of segment_sum / segment mean with respect to its data.
 * dgfx_batch_csr: the merged batch of a one-node-set, one-edge-set sampler
 * (dgfx_sampler_sample) as a CSR over batch nodes: row = batch index of an
 * edge's source, column (int32) = batch index of its target; rows past the
 * batch's node count up to node_capacity are empty (rowptr has
 * node_capacity + 1 entries), so no host synchronisation is needed. With
 * dgfx_spmm_csr(normalize=1) it is the mean aggregation of hetero_gnn.py:
 * 282-294 over the sampled subgraph, messages flowing from the sampled
 * neighbours to the node that sampled them.
 * ------------------------------------------------------------------------ */
int dgfx_csr_add_diagonal(const int64_t* d_rowptr, const int32_t* d_col, int64_t num_rows, float diag,
                          int32_t normalize_symmetric, int64_t* d_out_rowptr, int32_t* d_out_col, float* d_out_val,
                          dgfx_stream stream);
int dgfx_csr_row_ids(const int64_t* d_rowptr, int64_t num_rows, int64_t* d_out, dgfx_stream stream);
int dgfx_segment_counts(const int64_t* d_ids, int64_t n, int64_t num_segments, int32_t* d_counts, dgfx_stream stream);
int dgfx_gather_rows_scaled(const void* d_src, int dtype, const int64_t* d_ids, int64_t n, int64_t num_segments,
                            int64_t feat, const int32_t* d_counts, void* d_out, dgfx_stream stream);
int dgfx_batch_csr(const int64_t* d_node_offsets, const int64_t* d_edge_offsets, const int64_t* d_edge_src,
                   const int64_t* d_edge_dst, int64_t num_seeds, int64_t node_capacity, int64_t* d_rowptr,
                   int32_t* d_col, dgfx_stream stream);
/* dgfx_batch_mean: the same mean aggregation in one pass (one warp per
 * sample): out[v] = mean of feats[u] over the batch edges v -> u (fp32 sums
 * in edge order), zero rows for nodes without edges; rows past the batch's
 * node count are not written. feats / out [node_capacity, feat] in batch
 * order, fp32 or bf16, rows a multiple of 16 bytes and 16-byte aligned. */
int dgfx_batch_mean(const int64_t* d_node_offsets, const int64_t* d_edge_offsets, const int64_t* d_edge_src,
                    const int64_t* d_edge_dst, int64_t num_seeds, int64_t node_capacity, const void* d_feats,
                    int dtype, int64_t feat, void* d_out, dgfx_stream stream);

/* Writes *d_node_total and *d_edge_total (for a merged batch: the last words
 * of its node and edge offsets) to out2[0], out2[1] in stream order, from
 * one thread on the GPU. out2 may be pinned host memory (a device address
 * under unified addressing): a host that fills it with -1 and polls it
 * learns a batch's sizes as soon as the batch is sampled, without a stream
 * synchronisation or a copy that would queue behind earlier device-to-host
 * copies, and can then issue the copies of exactly those sizes. No reference
 * counterpart (the reference's batches live in host memory). */
int dgfx_publish_totals(const int64_t* d_node_total, const int64_t* d_edge_total,
                        int64_t* out2, dgfx_stream stream);

/* Copies up to two inputs into a captured CUDA graph's static buffers
 * (cudaMemcpyAsync, any direction under unified addressing; a zero size
 * skips a copy) and launches the graph exec, all in `stream` order: one call
 * per replay of a captured sampling step, so a caller issuing one batch per
 * replay pays one foreign call instead of a stream join, two tensor copies
 * and a replay. graph_exec is a cudaGraphExec_t. No reference counterpart
 * (the reference samples on the host). */
int dgfx_graph_launch_with_inputs(void* graph_exec, void* dst0, const void* src0, size_t bytes0, void* dst1,
                                  const void* src1, size_t bytes1, dgfx_stream stream);

/* ------------------------------------------------------------------------
 * Seeded synthetic inputs (stand-ins for the benchmark datasets, the role of
 * the reference's dgf/src/util/gen_test_graph.py generators at scale).
 * dgfx_synth_graph: power-law out-degrees (P(d) ~ d^-alpha, capped at
 * max_degree, rescaled to exactly num_edges), power-law target popularity;
 * writes rowptr int64[num_nodes + 1] and, if non-NULL, the source-major edge
 * list src/dst int64[num_edges]. Pure function of its arguments.
 * dgfx_synth_bipartite: the same with sources [0, num_src) and targets
 * drawn from [0, num_dst) (an edge type between two node sets; workspace as
 * dgfx_synth_graph_workspace_size(num_src, max_degree)).
 * dgfx_synth_uniform_int: out[i] uniform in [lo, hi) (Philox stream id).
 * dgfx_synth_normal_features: rows [node_begin, node_begin + count) of a
 * N(0,1) [*, dim] matrix keyed by node id (partition independent).
 * ------------------------------------------------------------------------ */
int dgfx_synth_graph_workspace_size(int64_t num_nodes, int64_t max_degree, size_t* bytes);
int dgfx_synth_graph(int64_t num_nodes, int64_t num_edges, double alpha,
                     int64_t max_degree, uint64_t seed, int64_t* d_rowptr,
                     int64_t* d_src, int64_t* d_dst, void* d_workspace,
                     size_t workspace_bytes, dgfx_stream stream);
int dgfx_synth_bipartite(int64_t num_src, int64_t num_dst, int64_t num_edges,
                         double alpha, int64_t max_degree, uint64_t seed,
                         int64_t* d_rowptr, int64_t* d_src, int64_t* d_dst,
                         void* d_workspace, size_t workspace_bytes,
                         dgfx_stream stream);
int dgfx_synth_uniform_int(int64_t n, int64_t lo, int64_t hi, uint64_t seed,
                           uint32_t stream_id, int64_t* d_out,
                           dgfx_stream stream);
int dgfx_synth_normal_features(int64_t node_begin, int64_t count, int64_t dim,
                               uint64_t seed, int dtype, void* d_out,
                               dgfx_stream stream);
/* dgfx_synth_normal_rows: the rows of the dgfx_synth_normal_features table
 * for an arbitrary list of node ids (regenerates any rank's rows, e.g. to
 * check rows gathered from peers). */
int dgfx_synth_normal_rows(const int64_t* d_ids, int64_t count, int64_t dim, uint64_t seed, int dtype, void* d_out,
                           dgfx_stream stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* DGFX_H_ */
