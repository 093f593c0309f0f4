/*
 * yanah_b200: C ABI of the B200 (sm_100a) sparse-MoE decode path.
 *
 * The reference engine (moe_prefetch) runs this path as MLX operations
 * called from Python (moe_prefetch/mlx_backend.py). Each entry point below
 * replaces one of those operation groups; the comment on each names the
 * reference call site (path:line inside the reference project).
 *
 * Conventions
 *  - Plain pointers and sizes only. Every pointer marked "device" is CUDA
 *    device memory of the current device; "host" pointers are host memory.
 *  - bf16 and fp16 values travel as uint16_t bit patterns.
 *  - Quantised matrices use MLX's affine format: `weight` is (rows,
 *    cols*bits/32) uint32 words, code k of a row sits in word k/(32/bits) at
 *    bit offset bits*(k%(32/bits)); `scales`/`biases` are (rows, cols/group)
 *    fp16; w[r][k] = scale*q + bias.
 *  - Expert records follow the repacked on-disk order gate/up/down x
 *    weight/scales/biases (moe_prefetch/repack.py:27-29), one record per slot.
 *  - Functions return 0 on success or a negative YN_E* code; nothing on the
 *    compute path allocates memory: callers pass a workspace sized by
 *    yn_workspace_bytes and cleared once with yn_workspace_init.
 *  - `stream` is a cudaStream_t passed as void*.
 */
#ifndef YANAH_B200_H
#define YANAH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- errors */
#define YN_OK 0
#define YN_E_INVALID (-1)      /* bad argument (shape, alignment, null pointer) */
#define YN_E_UNSUPPORTED (-2)  /* shape/bit-width outside what the kernels implement */
#define YN_E_CUDA (-3)         /* a CUDA runtime call failed (see yn_last_error) */
#define YN_E_DEVICE (-4)       /* a kernel reported an error in the workspace error word */

/* Text of the last error raised on this thread. */
const char* yn_last_error(void);

/* ------------------------------------------------------------ data types */

/* One MLX-affine quantised matrix (device pointers). */
typedef struct yn_qmat {
  const void* weight;   /* (rows, cols*bits/32) uint32 */
  const void* scales;   /* (rows, cols/group_size) fp16 */
  const void* biases;   /* (rows, cols/group_size) fp16 */
  int32_t rows, cols, bits, group_size;
} yn_qmat;

/* Model dimensions of one MoE layer (moe_prefetch/layout.py:28-40). */
typedef struct yn_dims {
  int32_t hidden;        /* H */
  int32_t n_experts;     /* E */
  int32_t top_k;         /* k */
  int32_t moe_inter;     /* I, routed expert intermediate size */
  int32_t shared_inter;  /* I_sh, shared expert intermediate size (0: none) */
  int32_t norm_topk;     /* 1: renormalise the top-k weights (norm_topk_prob) */
  float rms_eps;         /* RMSNorm epsilon */
} yn_dims;

/* Record geometry of one routed expert (moe_prefetch/repack.py:32-63). */
typedef struct yn_record {
  int32_t bits, group_size;
  int64_t piece_offset[9];  /* byte offset of each piece inside a record */
  int64_t record_bytes;
} yn_record;

/* Dense (resident) weights of one layer plus its routed-expert storage. */
typedef struct yn_layer {
  const void* post_norm;       /* (H) bf16 post_attention_layernorm weight */
  yn_qmat router;              /* (E, H) mlp.gate */
  const float* router_bias;    /* (E) fp32 logit offset added before softmax, or NULL */
  yn_qmat shared_gate;         /* (I_sh, H) shared_expert.gate_proj */
  yn_qmat shared_up;           /* (I_sh, H) shared_expert.up_proj */
  yn_qmat shared_down;         /* (H, I_sh) shared_expert.down_proj */
  yn_qmat shared_expert_gate;  /* (1, H) shared_expert_gate */
  const void* expert_base;     /* device base of the slot arena */
  int64_t slot_stride;         /* bytes between consecutive slots */
  int32_t n_slots;             /* slots addressable from expert_base */
  const int32_t* expert_slot;  /* (E) device table expert id -> slot, or NULL for slot = id */
  yn_record record;            /* routed expert record geometry */
} yn_layer;

/* ------------------------------------------------------------- workspace */

/* Bytes of workspace for one model shape. One workspace serves every call
 * (any row count T <= YN_MAX_ROWS, up to YN_MAX_TARGETS lookahead routers)
 * but calls that share a workspace must not run concurrently. */
#define YN_MAX_ROWS 8
#define YN_MAX_TARGETS 2
size_t yn_workspace_bytes(const yn_dims* dims);
/* Zero the workspace counters and error word (once, after allocation). */
int yn_workspace_init(void* ws, size_t ws_bytes, const yn_dims* dims, void* stream);
/* Read and clear the device error word (synchronises the stream). */
int yn_workspace_error(void* ws, const yn_dims* dims, void* stream, int32_t* code_out);

/* Device pointers to the named outputs inside a workspace (for readback).
 * Row t of a (T, ...) array starts at row t regardless of T. */
typedef struct yn_ws_view {
  void* x;         /* (T, H) bf16: post-attention RMSNorm output */
  float* logits;   /* (T, E) router logits (bf16 values held in fp32) */
  int32_t* ids;    /* (T, k) routed expert ids, descending probability */
  float* weights;  /* (T, k) routing weights (bf16 values held in fp32) */
  float* flogits;  /* (n_targets, T, E) lookahead router logits (bf16 values in fp32) */
  float* fprobs;   /* (n_targets, E) lookahead probabilities, max over rows */
  void* act;       /* (T, k, I) bf16 SwiGLU activations of the routed experts */
  void* act_sh;    /* (T, I_sh) bf16 SwiGLU activations of the shared expert */
  float* sgate;    /* (T) sigmoid(shared_expert_gate(x)), bf16 values */
  void* y;         /* (T*k, H) bf16 routed down outputs, row t*k + j */
  void* y_shared;  /* (T, H) bf16 sigmoid(gate) * shared down output */
  int32_t* error;  /* device error word */
} yn_ws_view;
int yn_workspace_view(void* ws, const yn_dims* dims, yn_ws_view* out);

/* --------------------------------------------------------------- kernels */

/* mx.dequantize (moe_prefetch/mlx_backend.py:272, quantize_2bit.py:158):
 * out[r][k] = fp32 fmaf(scale, q, bias), written as fp32 (rows, cols). */
int yn_dequantize(const yn_qmat* m, float* out, void* stream);

/* QuantizedLinear forward for T rows (mlx_backend.py:305-306, `m.gate(x)`):
 * y[t][r] = bf16(sum_k x[t][k] w[r][k]) in the canonical reduction order. */
int yn_qlinear(const yn_qmat* m, const void* x, int32_t T, float* y, void* stream);

/* Routing (mlx_backend.py:308-316): softmax(precise) -> top-k -> renormalise.
 * logits (T,E) fp32 holding bf16 values. ids (T,k) int32 in descending
 * probability (ties: lower id first); weights (T,k) bf16 values in fp32. */
int yn_route(const float* logits, int32_t T, const yn_dims* dims, int32_t* ids, float* weights,
             void* stream);

/* The post-attention half of a decoder layer plus routing and lookahead
 * (mlx_backend.py:302-306 `_post_attention` + :326-348 `route_and_forecast`):
 * x = RMSNorm(h1); shared-expert activations and gate; router logits; top-k
 * ids and weights; for each target layer t: softmax(router_t(RMSNorm_t(h1)))
 * in fp32, max over rows. All outputs land in the workspace (yn_ws_view). */
int yn_post_attention(const yn_dims* dims, const yn_layer* layer, const void* h1, int32_t T,
                      const yn_layer* targets, int32_t n_targets, void* ws, void* stream);

/* Routed-expert gate/up + SwiGLU for a subset of the k columns
 * (mlx_backend.py:447-456 `_switch_glu` up to swiglu; :376-391 `moe_ready`
 * starts the resident columns). ids: (T,k) device, or NULL to use the ids in
 * the workspace. cols: host array of column indices (NULL = all k). */
int yn_moe_up(const yn_dims* dims, const yn_layer* layer, const void* x, const int32_t* ids,
              int32_t T, const int32_t* cols, int32_t n_cols, void* ws, void* stream);

/* Down projections of every routed column and the shared expert, then the
 * combine (mlx_backend.py:456-459 down, :409/:420 weighted sum, :438-440
 * routed + shared, orchestrator.py:287 residual):
 *   mode 0: out = sum_j w_j y_j
 *   mode 1: out = sum_j w_j y_j + sigmoid(g) * shared(x)
 *   mode 2: out = h_res + (sum_j w_j y_j + sigmoid(g) * shared(x))
 * ids/weights: (T,k) device or NULL for the workspace's. out: (T,H) bf16. */
int yn_moe_down(const yn_dims* dims, const yn_layer* layer, const int32_t* ids, const float* weights,
                int32_t T, const void* h_res, int32_t mode, void* out, void* ws, void* stream);

/* One whole pool-path MoE layer on device (orchestrator.py:226-300 with every
 * expert resident): post_attention, routing, experts, combine, residual.
 * h_in/h_out: (T,H) bf16 device (may not alias). */
int yn_moe_layer(const yn_dims* dims, const yn_layer* layer, const void* h_in, int32_t T,
                 const yn_layer* targets, int32_t n_targets, void* h_out, void* ws, void* stream);

/* yn_moe_layer without a caller workspace: no counterpart in the reference
 * (its MLX backend allocates lazily). For callers that cannot allocate device
 * memory at call time or hand one over: an FFI binding (cgo, ctypes, JNI)
 * that owns no device allocator, or a process that has already given all free
 * HBM to the expert slot pool, where a cudaMalloc would fail or fragment it.
 * Nothing is allocated: the workspace is a file-scope device array of
 * YN_NOALLOC_SCRATCH_BYTES per device (yn_workspace_bytes(dims) larger than
 * that returns YN_E_UNSUPPORTED with the two sizes in yn_last_error).
 * The first call on each device looks up the array's address and zeroes it
 * with cudaMemsetAsync on `stream`; make that first call before any stream
 * capture. The error word and the combine counters at the front of the
 * workspace must start at zero: the counters return to zero at the end of
 * every call, the error word stays set until yn_workspace_error clears it, and
 * a call whose counter region reaches further than the last call's zeroes the
 * extension first. All calls share the one array per device: calls that
 * overlap in time (different streams, host threads without ordering) race and
 * give wrong results. scratch_out (optional) receives the array's device
 * address, for yn_workspace_view / yn_workspace_error. */
#define YN_NOALLOC_SCRATCH_BYTES (1u << 20)
int yn_moe_layer_noalloc(const yn_dims* dims, const yn_layer* layer, const void* h_in, int32_t T,
                         const yn_layer* targets, int32_t n_targets, void* h_out, void* stream,
                         void** scratch_out);

/* ------------------------------------------------ whole-stack bs1 decode */

/* Persistent decode of `n_tokens` sequential bs1 tokens through `n_layers`
 * resident MoE layers (orchestrator.py:308-343 with every expert resident):
 * one cooperative launch, one CTA per SM, three grid barriers per layer.
 * Prepare once: yn_stack_prepare copies the layer descriptors into a device
 * table of yn_stack_table_bytes(n_layers) bytes; `layers` is the same host
 * array (used for sizing). inputs/outputs: (n_tokens, H) bf16.
 * Per-layer traces, each optional (NULL: not written): trace_ids (n_tokens,
 * n_layers, k) routed ids; trace_hidden (n_tokens, n_layers, H) bf16, the
 * input row of every layer (16-byte aligned); trace_weights (n_tokens,
 * n_layers, k) fp32 routed weights. With them a caller can check every
 * layer of the decode against its own reference on the kernel's own layer
 * inputs. timing: (n_layers, 16, n_SMs) int64 global-timer stamps (ns) of the
 * last token's phases on every CTA, or NULL (diagnostics: adds a block sync
 * per stamp). */
size_t yn_stack_table_bytes(int32_t n_layers);
size_t yn_stack_scratch_bytes(const yn_dims* dims);
int yn_stack_prepare(const yn_dims* dims, const yn_layer* layers, int32_t n_layers, void* table, size_t table_bytes);
int yn_stack_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                    const void* inputs, int32_t n_tokens, void* outputs, void* scratch, size_t scratch_bytes,
                    int32_t* trace_ids, void* trace_hidden, float* trace_weights, int64_t* timing,
                    void* stream);
/* The same decode (same arguments, same results bit for bit) in data-flow
 * form: no grid barriers. The layer's work is split by routed column (groups
 * of CTAs that each compute gate/up and then down for one routed expert,
 * exchanging only that expert's activations) and every exchange between CTAs
 * is a set of flagged words read directly by its consumers: router logits,
 * the expert's activations, the shared expert's activations, the expert
 * outputs of a block of rows, the layer output. No counterpart in the
 * reference (a persistent-kernel schedule of orchestrator.py:308-343 with
 * every expert resident). scratch: yn_stack_flow_scratch_bytes(dims). */
size_t yn_stack_flow_scratch_bytes(const yn_dims* dims);
int yn_stack_flow_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                         const void* inputs, int32_t n_tokens, void* outputs, void* scratch, size_t scratch_bytes,
                         int32_t* trace_ids, void* trace_hidden, float* trace_weights, int64_t* timing,
                         void* stream);
/* Read and clear the stack decode error word (synchronises the stream);
 * either form's scratch. */
int yn_stack_error(void* scratch, const yn_dims* dims, void* stream, int32_t* code_out);
/* A batch of n_rows <= 8 token rows through every layer in one persistent
 * cooperative launch, in data-flow form: the forward of a speculative-verify
 * pass (moe_prefetch/speculative.py:121-193 runs the 1 + depth rows of a
 * draft through the model and compares; here its MoE part) and small decode
 * batches, every expert resident. Per layer each routed expert of the
 * batch (the union over its rows, ascending id) is read from HBM once by a
 * group of CTAs, its rows being the columns of the GEMV
 * (mlx_backend.py:411-436 moe over a batch's experts, :442-459 the expert
 * MLP); routing of every row is bit-identical to yn_post_attention
 * (mlx_backend.py:308-316). Compiled for hidden 2048, 64 experts, intermediate
 * 1536, top_k <= 8, 4-bit g64 routed experts, 8-bit g64 router, no shared
 * expert (the LFM2-24B-A2B shape); other shapes return YN_E_UNSUPPORTED.
 * table: yn_stack_prepare. inputs / outputs: (n_rows, hidden) bf16.
 * scratch: yn_rows_flow_scratch_bytes(dims, max_rows) for n_rows <= max_rows
 * (error word first: yn_stack_error reads it). trace_ids / trace_weights:
 * (n_layers, n_rows, k); trace_hidden: (n_layers, n_rows, hidden) each
 * layer's input rows; timing: (n_layers, 16, n_SMs) global-timer stamps;
 * each may be NULL. */
size_t yn_rows_flow_scratch_bytes(const yn_dims* dims, int32_t max_rows);
int yn_rows_flow_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                        const void* inputs, int32_t n_rows, void* outputs, void* scratch, size_t scratch_bytes,
                        int32_t* trace_ids, void* trace_hidden, float* trace_weights, int64_t* timing,
                        void* stream);

/* ------------------------------------- batch decode, expert parallelism */

/* A batch of T = n_ranks * rows_per_rank token rows (at most 64) through
 * one MoE layer with the routed experts grouped by expert, so each expert
 * record is read once per layer however many rows chose it
 * (mlx_backend.py:411-436 `moe` with :111-123 `_gather_sort`;
 * orchestrator.py:361-405 `generate_batch`). Expert parallelism has no
 * counterpart in the reference (one MLX device): rank r holds the routed
 * experts [expert_lo, expert_hi) of every layer in its arena (slot =
 * expert_slot[e], or e - expert_lo without a table) and rows
 * [r * rows_per_rank, (r+1) * rows_per_rank) of the batch ("home rows").
 * With n_ranks = 1 this is the single-GPU batch path. */
typedef struct yn_ep_config {
  int32_t rank, n_ranks, rows_per_rank;
  int32_t expert_lo, expert_hi;
  int32_t n_layers;  /* layers per step (the per-step flag and counter targets) */
} yn_ep_config;

/* Per rank two buffers: a peer-visible one of yn_ep_sym_bytes (gather rows,
 * flags, the home rows' routed outputs and their counter; every rank maps
 * every other rank's, see yn_ipc_export) and a private one of
 * yn_ep_local_bytes. Zero both once with yn_ep_init before the first layer
 * (all ranks, before any rank's first yn_ep_layer). */
size_t yn_ep_sym_bytes(const yn_dims* dims, const yn_ep_config* cfg);
size_t yn_ep_local_bytes(const yn_dims* dims, const yn_ep_config* cfg);
int yn_ep_init(void* sym, void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream);

/* One layer for this rank's home rows h_in -> h_out ((rows_per_rank, H)
 * bf16): post-attention and routing of the home rows, the rows and their ids
 * written into every rank's gather buffer (peer stores + a release flag),
 * the shared expert of the home rows, then (after every rank's flag) the
 * pairs of the local experts: gate/up + SwiGLU and the down projection, whose
 * output rows are stored into the home rank's buffer with a release counter,
 * and finally the combine of the home rows in column order plus the shared
 * expert and the residual. peer_sym: n_ranks device pointers, peer_sym[r] =
 * rank r's peer-visible buffer as mapped in this process (own buffer at
 * [rank]). Waits on other ranks are bounded (2 s): a timeout sets the error
 * word (yn_ep_error) and the remaining kernels of the step skip their work.
 * Call yn_ep_step_end after the last layer of every step (all ranks run the
 * same number of steps). Launches only kernels: capturable in a graph. */
int yn_ep_layer(const yn_dims* dims, const yn_layer* layer, int32_t layer_index, const yn_ep_config* cfg,
                const void* h_in, void* h_out, void* const* peer_sym, void* local, void* stream);
int yn_ep_step_end(void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream);
/* Read and clear the error word (synchronises the stream). */
int yn_ep_error(void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream, int32_t* code_out);

/* Device pointers into the buffers, for readback. */
typedef struct yn_ep_local_ptrs {
  void* x;          /* (rows_per_rank, H) bf16 normalised home rows */
  int32_t* ids;     /* (rows_per_rank, k) routed ids */
  float* weights;   /* (rows_per_rank, k) routing weights */
  void* act_sh;     /* (rows_per_rank, I_sh) shared-expert activations */
  float* sgate;     /* (rows_per_rank) shared-expert gate */
  void* y_shared;   /* (rows_per_rank, H) gated shared-expert outputs */
  int32_t* error;
  uint64_t* epoch;  /* steps completed */
} yn_ep_local_ptrs;
typedef struct yn_ep_sym_ptrs {
  void* x_all;        /* (n_ranks * rows_per_rank, H) gathered rows */
  int32_t* ids_all;   /* (n_ranks * rows_per_rank, k) */
  void* y;            /* (rows_per_rank, k, H) routed outputs of the home rows */
  uint64_t* flags;    /* (8, 16) arrival stamps: [writing rank][dispatch CTA] */
  uint64_t* counter;  /* finished (pair, 64-row tile) units, cumulative */
} yn_ep_sym_ptrs;
int yn_ep_view(void* local, const yn_dims* dims, const yn_ep_config* cfg, yn_ep_local_ptrs* out);
int yn_ep_sym_view(void* sym, const yn_dims* dims, const yn_ep_config* cfg, yn_ep_sym_ptrs* out);

/* Device memory for the peer-visible buffer (cudaMalloc, so that it can be
 * exported) and its CUDA IPC handle (YN_IPC_HANDLE_BYTES bytes) for the other
 * ranks' processes; import maps a peer's buffer with peer access enabled. */
#define YN_IPC_HANDLE_BYTES 64
int yn_device_alloc(size_t bytes, void** ptr);
int yn_device_free(void* ptr);
int yn_ipc_export(const void* dev_ptr, void* handle_out);
int yn_ipc_import(const void* handle, void** dev_ptr_out);
int yn_ipc_close(void* dev_ptr);
/* Copy between any host/device addresses (cudaMemcpyDefault), then wait for
 * `stream`: readback for callers that hold raw device pointers. */
int yn_memcpy(void* dst, const void* src, size_t bytes, void* stream);
/* The same copy, ordered on `stream` and not waited for (pinned host memory
 * for an asynchronous host<->device transfer). */
int yn_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);

/* -------------------------------------------- prefill: tensor-core GEMM */

/* Prompt prefill moves hundreds of rows through each expert (sweep.py:80-138
 * and the prompt pass of mlx_backend.py:421-433 `moe`), so the routed
 * experts run as a grouped GEMM on the tcgen05 tensor cores. The grouping
 * (which rows go to which expert) is planned by yn_prefill_plan on the
 * device, or by the caller.
 *
 * yn_rows_route: post-attention RMSNorm, router logits, top-k ids and
 * weights of T rows (T <= 4096), bit-identical to yn_post_attention row by
 * row; x_out (T, H) bf16 normalised rows. ws: yn_rows_route_bytes(dims,
 * max_rows) bytes for calls of up to max_rows rows, zeroed once before first
 * use; yn_route_error reads and clears its error word. */
size_t yn_rows_route_bytes(const yn_dims* dims, int32_t max_rows);
int yn_rows_route(const yn_dims* dims, const yn_layer* layer, const void* h, int32_t T, void* x_out,
                  int32_t* ids_out, float* w_out, void* ws, size_t ws_bytes, void* stream);
int yn_route_error(void* ws, const yn_dims* dims, void* stream, int32_t* code_out);

/* bf16 rows -> fp16 rows in the K-permuted order the tensor-core GEMM reads
 * (within each block of 8, element p at 2p for p < 4, at 2(p - 4) + 1 else). */
int yn_to_f16_kperm(const void* x, int64_t rows, int32_t cols, void* out, void* stream);

/* One tile of the grouped GEMM: expert e, pairs [p0, p0 + n) (n <= 256, the
 * pairs of one expert), first gate/up unit (mode 0, 64 units per tile) or
 * first output row (mode 1, 128 rows per tile). */
typedef struct yn_tc_tile {
  int32_t e, p0, n, u0;
} yn_tc_tile;

/* mode 0 (mlx_backend.py:447-456 `_switch_glu` up to SwiGLU): for every tile,
 * act_out[p][kperm(u)] = bf16(swiglu(gate_u . x_p, up_u . x_p)) with x_p =
 * b_rows[p] (fp16 K-permuted rows of H in pair order, yn_gather_f16_kperm;
 * weights dequantised to fp16). mode 1 (the down projection): y_out[p][h] =
 * bf16(down_h . act_p) with act_p = b_rows[p] (bf16 K-permuted rows of I;
 * weights dequantised to bf16). b_rows holds n_rows rows (read through TMA
 * tensor maps; 16-byte aligned). Routed experts 4-bit g64 only. tiles:
 * device array. err: device error word (bounded waits, bad slots). */
int yn_tc_experts(const yn_dims* dims, const yn_layer* layer, int32_t mode, const yn_tc_tile* tiles,
                  int32_t n_tiles, const int32_t* n_tiles_dev, const void* b_rows, int64_t n_rows,
                  void* act_out, void* y_out, int32_t* err, void* stream);
/* The gate/up GEMM's rows in pair order: out[p] = fp16 K-permuted copy of
 * x[row_of[p]] (bf16 rows of `cols`). */
int yn_gather_f16_kperm(const void* x, const int32_t* row_of, int64_t rows, int32_t cols, void* out, void* stream);

/* The grouping on the device, so that a prefill layer needs no host
 * synchronisation: pairs of each expert made contiguous (pair_row: pair ->
 * row, pair_of: t * k + j -> pair), then the gate/up and down tiles of every
 * expert (n_tiles[0], n_tiles[1] on the device; pass them to yn_tc_experts
 * as n_tiles_dev with grids of max_up / max_dn from yn_prefill_max_tiles). */
int yn_prefill_max_tiles(const yn_dims* dims, int32_t T, int32_t* max_up, int32_t* max_dn);
int yn_prefill_plan(const yn_dims* dims, const int32_t* ids, int32_t T, int32_t* pair_row, int32_t* pair_of,
                    yn_tc_tile* tiles_up, int32_t max_up, yn_tc_tile* tiles_dn, int32_t max_dn, int32_t* n_tiles,
                    int32_t* err, void* stream);

/* Combine of T rows (mlx_backend.py:409/:420, :438-440; orchestrator.py:287):
 * out[t] = h_res[t] + (sum_j bf16(y[pair_of[t][j]] * w[t][j]) in column order
 * + y_shared[t]); y_shared and h_res may be NULL. Columns whose pair_of entry
 * is negative are skipped (a staging group of the prefill sweep computes only
 * the pairs of its experts, mlx_backend.py:421-433). */
int yn_pairs_combine(const yn_dims* dims, const void* y, const int32_t* pair_of, const float* weights,
                     const void* y_shared, const void* h_res, int32_t T, void* out, void* stream);

/* Rows (row_of[p], or p when row_of is NULL) of x (bf16, cols % 16 == 0) in the
 * K order the tensor-core GEMM uses for `bits`-bit codes (2, 4 or 8), as fp16
 * (f16 != 0, gate/up operands) or bf16 (down operands). The 4-bit order is
 * yn_gather_f16_kperm's. Part of the prompt pass of sweep.py:80-138 /
 * mlx_backend.py:421-433 for every record format. */
int yn_gather_kperm(const void* x, const int32_t* row_of, int64_t rows, int32_t cols, int32_t bits, int32_t f16,
                    void* out, void* stream);
/* out[t][c] = bf16(scale[t] * y[t][c]) for bf16 y: the gated shared-expert term
 * sigmoid(g) * shared(x) of many rows (mlx_backend.py:302-306 with :438-440). */
int yn_scale_rows(const void* y, const float* scale, int64_t rows, int32_t cols, void* out, void* stream);
/* Where yn_rows_route of T rows left the shared expert's SwiGLU activations
 * (T, shared_inter) bf16 and its gates sigmoid(g) (T) fp32 in `ws`. */
int yn_rows_route_shared(const yn_dims* dims, int32_t T, void* ws, void** act_sh, float** sgate);

/* ---------------------------------------------------------- slot copies */

/* Copy `n` expert records host -> slot arena (io_lanes.py:121-126
 * read_record, which the reference runs as preadv into pool slots):
 * record i goes from host_src[i] (pinned host memory recommended) to
 * arena + slot[i]*slot_stride. One cudaMemcpyAsync per record on `stream`. */
int yn_slot_copy(void* arena, int64_t slot_stride, const int32_t* slots, const void* const* host_src,
                 int32_t n, int64_t record_bytes, void* stream);

/* ------------------------------------------------------- synthetic data */

/* Fill `n_words` uint32 words with the counter-based generator used for the
 * seeded synthetic workloads: word i = hash(seed, stream_id, i). */
int yn_synth_u32(void* dst, int64_t n_words, uint64_t seed, uint64_t stream_id, void* stream);
/* Fill `n` fp16 values with approximately normal samples (Irwin-Hall, 4
 * uniforms) of standard deviation `std` (absolute value if `absolute`). */
int yn_synth_f16(void* dst, int64_t n, uint64_t seed, uint64_t stream_id, float std, int32_t absolute,
                 void* stream);
/* Same for bf16 outputs. */
int yn_synth_bf16(void* dst, int64_t n, uint64_t seed, uint64_t stream_id, float std, float mean,
                  void* stream);

/* Record a CUDA timing event (cudaEvent_t as void*) on `stream`. While the
 * stream is being captured into a CUDA graph the record is captured as an
 * external event node, so kernel durations can be read per graph replay.
 * Benchmark instrumentation; no counterpart in the reference. */
int yn_record_event(void* event, void* stream);
/* Create / destroy a timing event; elapsed milliseconds between two records. */
int yn_event_create(void** event);
int yn_event_destroy(void* event);
int yn_event_elapsed_ms(void* start, void* end, float* ms);

/* Library version string. */
const char* yn_version(void);

#ifdef __cplusplus
}
#endif
#endif /* YANAH_B200_H */
