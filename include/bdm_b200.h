/*
 * bdm_b200.h -- C ABI of the B200-native Block Delta Memory (BDM) layer hot path.
 *
 * Plain pointers and sizes only.  Every device pointer is memory the caller
 * owns (PyTorch allocations in the bundled Python module); the library
 * allocates nothing.  Every call is asynchronous on the given CUDA stream
 * (`stream` is a cudaStream_t passed as void*, NULL = legacy default stream)
 * and returns a status code; BDM_ERR_CUDA means a launch failed (details in
 * bdm_last_cuda_error()).  Kernels never trap: an index read from memory that
 * is out of range is skipped and counted in the optional device error word.
 *
 * Element types: BDM_F32 (float) and BDM_BF16 (__nv_bfloat16, RNE rounding).
 * Index tensors are int64, as in the reference.
 *
 * Tensor layouts (row-major, contiguous unless a leading dimension `ld*` is
 * given):  NT = batch*time tokens, H heads, S = bank_size rows per bank,
 * dv = head_value_width, V = H*dv, KW / KR = write / read banks per token.
 *   q, k, b    [NT, H, S]  activation dtype        g [NT, H, S] float
 *   v, w       [NT, V]     activation dtype
 *   routes     write_idx/write_w [NT, KW], read_idx/read_w [NT, KR]
 *   bank state [batch, J, H, S, dv] (H = 1 is the reference's [batch, J, S, V])
 *   reads      [NT, KR, V] read output of every read event, by route slot
 *
 * Each entry point names the reference interface it replaces
 * (p0rc314in/bdm, implementation/bdm/<file>:<lines>).
 */
#ifndef BDM_B200_H
#define BDM_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define BDM_API __attribute__((visibility("default")))
#else
#define BDM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum bdm_status {
    BDM_OK = 0,
    BDM_ERR_INVALID = 1,     /* bad size, shape or null pointer */
    BDM_ERR_DTYPE = 2,       /* unsupported element type */
    BDM_ERR_UNSUPPORTED = 3, /* geometry outside what the kernels implement */
    BDM_ERR_CUDA = 4,        /* a CUDA call failed; see bdm_last_cuda_error() */
    BDM_ERR_WORKSPACE = 5    /* workspace missing or too small */
};

enum bdm_dtype { BDM_F32 = 0, BDM_BF16 = 1 };

/* Human-readable status text (static storage). */
/* *dst |= *src (device ints) as an atomic OR on `stream`: folds a launch's error bits into a word
 * that launches on other streams may update at the same time.  Utility; no reference counterpart. */
BDM_API int bdm_status_or(int *dst, const int *src, void *stream);
BDM_API const char *bdm_status_string(int status);
/* cudaError_t of the last call that returned BDM_ERR_CUDA on this host thread. */
BDM_API int bdm_last_cuda_error(void);
/* ABI revision of this header. */
BDM_API int bdm_abi_version(void);
/* Kernels launched by this library since it was loaded (all threads). */
BDM_API long long bdm_kernel_launches(void);

/*
 * Product-key top-B routing.  Replaces product_key_route
 * (gdn2_banks.py:74-114), also in its batch_factors form (gdn2_banks.py:93-102).
 *   logits  [ntok, ld] (dtype); factor scores at columns [0, j1) and [j1, j1+j2)
 *   indices [ntok, count] int64, weights [ntok, count] (dtype), count = min(selected, sub^2),
 *   sub = min(selected, j1, j2).  Ordered by descending pair score; ties go to
 *   the lower index at both top-k stages.  Pair scores are summed in the
 *   logits dtype; the softmax is FP32 and rounded to dtype.
 */
BDM_API int bdm_route(const void *logits, int64_t ntok, int64_t ld, int j1, int j2, int selected, int dtype,
              int64_t *indices, void *weights, void *stream);

/*
 * Two product-key routers over the same rows in one launch (the layer's write
 * router at columns [0, j1+j2) and read router at [second, second+j1+j2) of the
 * fused projection): results as two bdm_route calls.  No reference counterpart
 * (the reference calls product_key_route once per role, gdn2_banks.py:74-114).
 */
BDM_API int bdm_route_pair(const void *logits, int64_t ntok, int64_t ld, int64_t second, int j1, int j2, int selected,
                           int dtype, int64_t *indices, void *weights, int64_t *indices2, void *weights2,
                           void *stream);

/*
 * Causal bank dispatch: a stable counting sort of all events by (batch, bank).
 * Replaces role_bank_dispatch.metadata (role_bank_dispatch.py:143-153: _keys,
 * torch.sort, _bounds) and the ordering of pack_bank_events
 * (gdn2_banks.py:174-185, 237-246).
 *   Event ids: write (token, slot) -> token*kw + slot; read -> NT*kw + token*kr + slot.
 *   order      [E] int64, E = NT*(kw+kr): event id at each packed position, sorted
 *              by ((batch*J + bank)*T + t)*2 + role; equal keys keep id order.
 *   cu_seqlens [batch*J + 1] int64.
 *   inverse    [E] int64 or NULL: packed position of each event id.
 *   tokens     [E] int64 or NULL: token of each packed position.
 *   error_word int32 device pointer or NULL: incremented for each out-of-range bank.
 * The workspace (device memory, bdm_dispatch_workspace_bytes) is scratch.
 */
BDM_API int64_t bdm_dispatch_workspace_bytes(int64_t batch, int64_t time, int kw, int kr, int64_t bank_count);
BDM_API int bdm_dispatch(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time, int kw, int kr,
                 int64_t bank_count, int64_t *order, int64_t *cu_seqlens, int64_t *inverse, int64_t *tokens,
                 int32_t *error_word, void *workspace, int64_t workspace_bytes, void *stream);

/*
 * bdm_dispatch for callers that cannot allocate device memory -- code running
 * under CUDA graph capture, runtimes that own every device allocation, or
 * request paths that must not allocate.  No counterpart in the reference.
 * Same arguments and results as bdm_dispatch minus the workspace: scratch is a
 * fixed 32 MiB array inside the library (held on every GPU that loads it until
 * exit).  Needs bdm_dispatch_workspace_bytes(...) <= 32 MiB, else returns
 * BDM_ERR_WORKSPACE.  The first call on a device looks the array up (make it
 * before any stream capture), and so does the first call after the device's
 * context was re-created (cudaDeviceReset).  Calls share the array: calls that
 * may overlap on the GPU race and must be ordered by the caller.
 */
BDM_API int bdm_dispatch_noalloc(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time,
                                 int kw, int kr, int64_t bank_count, int64_t *order, int64_t *cu_seqlens,
                                 int64_t *inverse, int64_t *tokens, int32_t *error_word, void *stream);

/*
 * Controller epilogue over the fused input projection.  Replaces the
 * element-wise part of _parameters._controllers (_parameters.py:189-220) and
 * heads.controllers (heads.py:11-22); the projections themselves are GEMMs
 * done by the caller: proj = hidden @ [Wq;Wk;Wv;Wf1;Wb;Ww;...]^T and
 * f = f1 @ Wf2^T (the second f_proj layer, rounded to dtype like the reference's Linear).
 *   proj [ntok, ld] (dtype) with the q, k, v, b, w blocks at the given column offsets
 *   f [ntok, ldf] (dtype, H*S columns); or f = NULL and wf2 [H*S, f1_width] (dtype, the
 *   second f_proj layer's weight): the kernel computes f = dtype(f1 @ wf2^T) itself from
 *   proj columns [col_f1, col_f1 + f1_width) (FP32 accumulation; meant for few tokens)
 *   a_log [H], dt_bias [H*S] float
 *   qk_norm: 0 = F.normalize (original), 1 = x*rsqrt(sum x^2 + 1e-6) (nvidia)
 *   out: q, k, b [ntok, H, S] (dtype), g [ntok, H, S] float, v, w [ntok, V] (dtype)
 */
BDM_API int bdm_controllers(const void *proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k, int64_t col_v,
                            int64_t col_b, int64_t col_w, const void *f, int64_t ldf, const void *wf2,
                            int64_t col_f1, int f1_width, const float *a_log,
                            const float *dt_bias, int heads, int bank_size, int head_value_width, int qk_norm,
                            int dtype, void *q, void *k, void *v, float *g, void *b, void *w, void *stream);

/*
 * Product-key initial bank memory.  Replaces materialize_initial_state
 * (_parameters.py:40-67) and product_routed_update.materialize
 * (product_routed_update.py:10-21).
 *   out[n, j, h, s, :] = round_param(U[r / Q] + Z[r % Q]),  r = (j*H + h)*S + s,
 *   U [P, dv], Z [Q, dv] in factor dtype; out [batch, J, H, S, dv] in out dtype.
 */
BDM_API int bdm_product_state(const void *row_factor, const void *col_factor, int64_t rows_p, int64_t cols_q,
                      int factor_dtype, int64_t batch, int64_t bank_count, int heads, int bank_size,
                      int head_value_width, void *out, int out_dtype, void *stream);

/*
 * Per-bank delta-rule recurrence over dispatched events (one pass over every
 * (batch, bank, head) sequence).  Replaces routed_update.RoutedUpdate.forward
 * -> role_bank_dispatch.pack + decay_transform + role_bank_kernel.forward
 * (routed_update.py:5-32, role_bank_dispatch.py:156-185, role_bank_kernel.py:46-73,177-202)
 * and, with a cache, inference._bank_prefill (inference.py:134-158).
 *
 * Per write event (token t, slot j, p = write_w[t,j]) and head h, in FP32:
 *   M <- diag(exp(g_e)) M ;  u = w_e * v - (b_e * k)^T M ;  M <- M + k u^T
 *   g_e = routed_decay ? g*p : g,  b_e = dtype(b*p),  w_e = dtype(w*p)
 * Per read event (token t, slot j, r = read_w[t,j]):
 *   reads[t*kr + j, h*dv:(h+1)*dv] = dtype(scale * M^T dtype(q*r))
 * Initial state: `cache` when non-NULL ([batch,J,H,S,dv], cache_dtype), else the
 * product-key factors (row_factor/col_factor as in bdm_product_state).
 * state_interval > 0 rounds the FP32 state to BF16 before every
 * state_interval-th event of a sequence and rounds the initial state
 * (gdn2_banks.py:33-36); 0 keeps FP32 throughout (prefill).
 * store_final writes the final state into `cache` (cache must be non-NULL).
 * bank_ids [bank_count] int32 or NULL: on a bank-sharded rank, the sequences are
 * (batch, local bank) and bank_ids maps a local bank to its bank in the full
 * table of total_banks banks (used for the product-key initial state); NULL
 * means local = global and total_banks is ignored.
 * head_offset, total_heads: the call's `heads` heads are heads
 * [head_offset, head_offset + heads) of a layer with total_heads heads (a head
 * group; only the product-key initial state depends on it).  total_heads = 0
 * means heads (and head_offset 0); a cache needs the whole layer.
 * workspace: device scratch of bdm_bank_scan_workspace_bytes(batch, bank_count)
 * bytes (the per-launch work list: non-empty sequences by length class, so
 * long sequences start first and empty ones cost nothing).  The int32 at byte
 * 128 of the workspace holds error bits after the kernel: 1 = a wait between
 * the staging warp and the state warps of a CTA gave up (bounded at ~2 s; the
 * CTA's outputs are then incomplete).
 * checkpoints (training; NULL otherwise): the state before every
 * checkpoint_block-th event (position > 0) of a sequence is written to
 * checkpoints[(start / checkpoint_block + seq + pos / checkpoint_block), head, S, dv]
 * (float), the layout bdm_scan_backward reads with checkpoints_ready = 1
 * (checkpoint_block = bdm_scan_backward_block_events(S, dv)); sequences of 2048 or
 * more events may run on the long-sequence kernel, which writes none.  Needs the
 * factor-initialised whole-layer form (no cache, bank_ids or head group).
 * Supported: bank_size in {4, 8, 16}; head_value_width a multiple of 8.
 */
BDM_API int64_t bdm_bank_scan_workspace_bytes(int64_t batch, int64_t bank_count);
BDM_API int bdm_bank_scan(const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                          const int64_t *write_idx, const void *write_w, const int64_t *read_idx, const void *read_w,
                          const int64_t *order, const int64_t *cu_seqlens, int64_t batch, int64_t time,
                          int64_t bank_count, int heads, int bank_size, int head_value_width, int kw, int kr,
                          int dtype, int routed_decay, float scale, const void *row_factor, const void *col_factor,
                          int64_t factor_cols, int factor_dtype, const int32_t *bank_ids, int64_t total_banks,
                          int head_offset, int total_heads, void *cache, int cache_dtype, int store_final,
                          int state_interval, void *reads,
                          void *workspace, int64_t workspace_bytes, float *checkpoints, int checkpoint_block,
                          void *stream);
/*
 * Diagnostics, no counterpart in the reference: makes the recurrence's bounded waits testable
 * without a GPU fault.  wait_ns (0 = the default 2 s) bounds the long-sequence kernel's
 * producer / consumer waits; fault = 1 makes its producer withhold each CTA's first batch
 * hand-off, so the consumers' wait runs out, they set BDM_SCAN_ERR_TIMEOUT (bit 1) in the
 * workspace status word and every warp returns.  Applies to bdm_bank_scan calls made after it,
 * process-wide; outputs of a call that timed out are unspecified.  bdm_scan_test_fault(0, 0)
 * restores normal operation.
 */
BDM_API int bdm_scan_test_fault(int fault, unsigned long long wait_ns);

/*
 * bdm_bank_scan with the sequences below the long-sequence bound run in chunks on the tensor
 * cores (tcgen05.mma kind::tf32, accumulators in tensor memory): per chunk of C events (the
 * reference's BF16 storage interval, role_bank_kernel.py:153: 16 for bank_size <= 8, 8 for 16)
 * U = (I + Z)^-1 (X - Y M0) and the state carry are tensor-core products; the inter-chunk state
 * stays in FP32 registers.  Same arguments, outputs and storage policy as bdm_bank_scan.
 * BF16 only, head_value_width a multiple of 128, state_interval 0 or C, no checkpoints;
 * anything else returns BDM_ERR_UNSUPPORTED.  Outputs agree with bdm_bank_scan within the BF16
 * tolerance (tf32 operands), not bit for bit.
 */
BDM_API int bdm_bank_scan_chunked(const void *q, const void *k, const void *v, const float *g, const void *b,
                                  const void *w, const int64_t *write_idx, const void *write_w,
                                  const int64_t *read_idx, const void *read_w, const int64_t *order,
                                  const int64_t *cu_seqlens, int64_t batch, int64_t time, int64_t bank_count,
                                  int heads, int bank_size, int head_value_width, int kw, int kr, int dtype,
                                  int routed_decay, float scale, const void *row_factor, const void *col_factor,
                                  int64_t factor_cols, int factor_dtype, const int32_t *bank_ids,
                                  int64_t total_banks, int head_offset, int total_heads, void *cache,
                                  int cache_dtype, int store_final, int state_interval, void *reads,
                                  void *workspace, int64_t workspace_bytes, float *checkpoints,
                                  int checkpoint_block, void *stream);

/*
 * Read combine + output normalisation + sigmoid gate.  Replaces
 * role_bank_dispatch.readout / scatter_bank_outputs (role_bank_dispatch.py:219-231,
 * gdn2_banks.py:265-283) and the normalisation and gate of _project_bank_output
 * (_parameters.py:222-232); the o_proj GEMM follows in the caller.
 *   reads [ntok, kr, width] (dtype) summed per token in ascending bank order of
 *   read_idx [ntok, kr]; round_each = 1 rounds to dtype after every add (GPU
 *   reference readouts), 0 accumulates in FP32 and rounds once (CPU reference).
 *   With read_idx == NULL, `reads` is an already combined [ntok, width] tensor.
 *   gate [ntok, ld_gate] (dtype): output_gate pre-activation including its bias.
 *   norm_mode 1 = LayerNorm(weight, bias, eps), 0 = RMS (weight, eps).
 *   out [ntok, width] (dtype) = dtype(norm(raw) * dtype(sigmoid(gate))).
 */
BDM_API int bdm_combine_norm_gate(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                          const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias,
                          float eps, int norm_mode, int round_each, int dtype, void *out, void *stream);
/* bdm_combine_norm_gate that also stores the combined read sum raw_out [ntok, width]
 * (dtype): the tensor the reference's readout returns (routed_update.py:28-29) and
 * its output backward consumes. */
BDM_API int bdm_combine_norm_gate_save(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                       const void *gate, int64_t ld_gate, const void *norm_weight,
                                       const void *norm_bias, float eps, int norm_mode, int round_each, int dtype,
                                       void *out, void *raw_out, void *stream);

/*
 * Read combine + output normalisation + sigmoid gate + output projection in one kernel: the
 * whole output interface of the layer forward.  Replaces _readout (role_bank_dispatch.py:201-216)
 * followed by _project_bank_output (_parameters.py:222-232: o_proj(norm(y) * sigmoid(gate)) + b).
 *   reads, read_idx, gate, norm_*, eps, norm_mode, round_each: as bdm_combine_norm_gate.
 *   o_weight [out_dim, width] (dtype, rows contiguous: nn.Linear.weight), o_bias [out_dim] or NULL.
 *   out [ntok, ld_out] (dtype) = o_proj(dtype(norm(raw) * dtype(sigmoid(gate)))) + o_bias, FP32
 *   accumulation, one rounding to dtype.  The normalised input of o_proj is bit-identical to
 *   bdm_combine_norm_gate's output and is never written to memory.
 *   status: optional device int; a bounded wait inside the kernel that gave up ORs in 0x2 (the
 *   outputs of that launch are then unspecified).
 * BF16 only, 512 <= width <= 1024 with width % 256 == 0, out_dim % 128 == 0 and <= 1024,
 * 1 <= kr <= 16, reads / gate / norm_* / o_weight / out 16-byte aligned, ld_gate and ld_out multiples
 * of 8; other shapes return BDM_ERR_UNSUPPORTED (run bdm_combine_norm_gate and a GEMM instead).
 * bdm_combine_project_supported: 1 when (width, out_dim, kr, dtype) fits, else 0 (no launch).
 */
BDM_API int bdm_combine_project(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias,
                                float eps, int norm_mode, int round_each, const void *o_weight, const void *o_bias,
                                int64_t out_dim, int dtype, void *out, int64_t ld_out, int *status, void *stream);
BDM_API int bdm_combine_project_supported(int64_t width, int64_t out_dim, int kr, int dtype);

/*
 * Training backward.  Replaces the backward passes of RoutedUpdate /
 * RoleBankTraining / ProductRoutedUpdate (routed_update.py:31-49,
 * role_bank_kernel.py:76-150,204-215, product_routed_update.py:44-76) and, for the
 * ops around them, the autograd of product_key_route (gdn2_banks.py:74-114),
 * _controllers (_parameters.py:189-220, heads.py:11-22) and _project_bank_output
 * (_parameters.py:222-232).  All gradients accumulate in FP32; tensors the
 * reference keeps in the parameter dtype are rounded to it at the same points.
 *
 * bdm_norm_gate_backward: d_out [ntok, width] (gradient of the o_proj input),
 *   raw [ntok, width] (from bdm_combine_norm_gate_save), gate [ntok, ld_gate]
 *   pre-activations -> d_raw [ntok, width], d_gate [ntok, ld_d_gate] (dtype) and
 *   the FP32 parameter gradients d_norm_weight [width], d_norm_bias [width]
 *   (LayerNorm with a bias only; may be NULL otherwise).  `partials` holds
 *   bdm_norm_gate_backward_partial_floats(ntok, width) floats.
 * bdm_scan_backward: the recurrence backward over the dispatched events (same
 *   inputs as bdm_bank_scan's factor-initialised training call, plus d_read
 *   [ntok, H*dv] = gradient of the combined read sum).  Outputs, FP32:
 *   event_grads [tiles, E, H, 3*S] per-(event, head) column sums (tiles =
 *   bdm_scan_backward_tiles(S, dv)) (per write event id:
 *   sum_x dh*u | sum_x hd*du | sum_x dh'*hd; per read event id: sum_x h*do),
 *   d_write_value [ntok*kw, H*dv] (du per write event id) and d_initial
 *   [batch*J, H, S, dv].  checkpoints: bdm_scan_backward_checkpoint_bytes() bytes
 *   holding the states at block starts; with checkpoints_ready = 1 the training forward
 *   (bdm_bank_scan with these checkpoints) already wrote them, except for sequences of
 *   2048 or more events, whose checkpoints this call replays itself.  S in {4, 8, 16}.
 * bdm_event_vjp: per-token gather of the event gradients (role_bank_dispatch.py:
 *   76-132 plus the routed-decay dp term of routed_update.py:43-47): dq, dk, db
 *   [ntok, H*S], dv, dw [ntok, H*dv] (dtype), dg [ntok, H*S] (float), and the route
 *   weight gradients of each head, d_write_w_heads [ntok, H, kw] and
 *   d_read_w_heads [ntok, H, kr] (dtype; the reference runs one routed update per
 *   head).  dv <= 256.
 * bdm_product_state_backward: d_initial [batch, P*Q, dv] -> d_rows [P*Q, dv]
 *   (per logical row, batch-summed) and the factor gradients d_row_factor [P, dv],
 *   d_col_factor [Q, dv] (FP32 holding factor-dtype values).
 * bdm_route_backward: both routers' backward over one projection [ntok, ld]:
 *   blocks at columns first and second (J1+J2 logits each), selections idx_* [ntok,
 *   count] and per-head weight gradients dw_* [ntok, heads, count] (dtype; summed
 *   over heads in ascending order) -> d_logits blocks of [ntok, ldd] (every logit of
 *   both blocks written).  count <= 32.
 * bdm_controllers_backward: q, k, v, b, w column blocks of d_proj [ntok, ldd]
 *   (dtype), df [ntok, H*S] (dtype; gradient of f_proj's output) and the FP32
 *   d_dt_bias [H*S], d_a_log [H], from the forward's proj, f, g, b, w and the
 *   control gradients.  `partials` holds
 *   bdm_controllers_backward_partial_floats(ntok, H, S) floats.
 */
BDM_API int64_t bdm_norm_gate_backward_partial_floats(int64_t ntok, int64_t width);
BDM_API int bdm_norm_gate_backward(const void *d_out, const void *raw, int64_t ntok, int64_t width, const void *gate,
                                   int64_t ld_gate, const void *norm_weight, const void *norm_bias, float eps,
                                   int norm_mode, int dtype, void *d_raw, void *d_gate, int64_t ld_d_gate,
                                   float *partials, float *d_norm_weight, float *d_norm_bias, void *stream);
/* Column tiles of bdm_scan_backward's event_grads (its leading dimension); -1 if unsupported. */
BDM_API int bdm_scan_backward_tiles(int bank_size, int head_value_width);
/* Events between the backward's state checkpoints (the checkpoint_block a training
 * forward passes to bdm_bank_scan); -1 if unsupported. */
BDM_API int bdm_scan_backward_block_events(int bank_size, int head_value_width);
BDM_API int64_t bdm_scan_backward_checkpoint_bytes(int64_t batch, int64_t time, int kw, int kr, int64_t bank_count,
                                                   int heads, int bank_size, int head_value_width);
BDM_API int bdm_scan_backward(const void *q, const void *k, const void *v, const float *g, const void *b,
                              const void *w, const void *write_w, const void *read_w, const int64_t *order,
                              const int64_t *cu_seqlens, int64_t batch, int64_t time, int64_t bank_count, int heads,
                              int bank_size, int head_value_width, int kw, int kr, int dtype, int routed_decay,
                              float scale, const void *row_factor, const void *col_factor, int64_t factor_cols,
                              int factor_dtype, int state_interval, const void *d_read, float *event_grads,
                              float *d_write_value, float *d_initial, float *checkpoints, int64_t checkpoint_bytes,
                              int checkpoints_ready, void *stream);
BDM_API int bdm_event_vjp(const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                          const void *write_w, const void *read_w, const float *event_grads,
                          const float *d_write_value, int64_t ntok, int heads, int bank_size, int head_value_width,
                          int kw, int kr, int dtype, int routed_decay, float scale, void *dq, void *dk, void *dv,
                          float *dg, void *db, void *dw, void *d_write_w_heads, void *d_read_w_heads,
                          void *stream);
BDM_API int bdm_product_state_backward(const float *d_initial, int64_t batch, int64_t rows_p, int64_t cols_q,
                                       int head_value_width, int factor_dtype, float *d_rows, float *d_row_factor,
                                       float *d_col_factor, void *stream);
BDM_API int bdm_route_backward(const void *logits, int64_t ntok, int64_t ld, int64_t first, int64_t second, int j1,
                               int j2, int count, int heads, const int64_t *idx_first, const void *dw_first,
                               const int64_t *idx_second, const void *dw_second, int dtype, void *d_logits,
                               int64_t ldd, void *stream);
BDM_API int64_t bdm_controllers_backward_partial_floats(int64_t ntok, int heads, int bank_size);
BDM_API int bdm_controllers_backward(const void *proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k,
                                     int64_t col_v, int64_t col_b, int64_t col_w, const void *f, int64_t ldf,
                                     const float *a_log, const float *dt_bias, const float *g, const void *b,
                                     const void *w, const void *dq, const void *dk, const void *dv, const float *dg,
                                     const void *db, const void *dw, int heads, int bank_size, int head_value_width,
                                     int qk_norm, int dtype, void *d_proj, int64_t ldd, void *df, float *partials,
                                     float *d_dt_bias, float *d_a_log, void *stream);

/*
 * Bank-sharded forward (one rank per GPU; no counterpart in the reference,
 * which runs the layer on one device).  The bank table is partitioned over
 * `world` ranks; each rank runs the recurrence of its own banks over the events
 * of all ranks' tokens and returns FP32 read partials.
 *
 * bdm_bank_histogram: counts[bank] += number of write and read events routed to
 *   it by write_idx [ntok, kw] and read_idx [ntok, kr] (int32 counts [bank_count],
 *   zeroed by the caller; out-of-range banks are clamped).
 * bdm_bank_owners: the partition.  mode 0 = contiguous index ranges
 *   (owner = bank / (J/world)); mode 1 = balanced by load: banks sorted by
 *   (count desc, index asc), then taken in groups of `world`; in the first 128
 *   groups the p-th heaviest bank of a group goes to the rank with the p-th
 *   smallest load (ties to the lower rank), later groups go in a serpentine
 *   over the ranks ordered by their load after group 128.  Both
 *   give every rank exactly J/world banks; J % world == 0 is required and mode 1
 *   needs J <= 16384 and world <= 32.  Outputs, int32: owner [J], slot [J] (the
 *   bank's index among its owner's banks, ascending bank order) and members
 *   [world, J/world] (members[r][slot] = bank).  Deterministic: equal counts give
 *   equal maps on every rank.
 * bdm_dispatch_owned: bdm_dispatch restricted to the banks with owner[bank] ==
 *   rank; sequence ids are batch*local_banks + slot[bank], cu_seqlens has
 *   batch*local_banks + 1 entries and cu_seqlens[batch*local_banks] is the owned
 *   event count.  `order` still lists every event: owned ones first (sorted as
 *   in bdm_dispatch), then the others.
 * bdm_combine_partial: out[t] = sum, in ascending bank order and FP32, of the
 *   read rows reads[t, j] (dtype) whose bank read_idx[t, j] this rank owns
 *   (out [ntok, width] float; zero where it owns none).
 * bdm_norm_gate_f32: bdm_combine_norm_gate over an FP32 combined read sum
 *   [ntok, width], rounded once to dtype first (the forward's round-once combine).
 */
BDM_API int bdm_bank_histogram(const int64_t *write_idx, const int64_t *read_idx, int64_t ntok, int kw, int kr,
                               int64_t bank_count, int32_t *counts, void *stream);
BDM_API int bdm_bank_owners(const int32_t *counts, int64_t bank_count, int world, int mode, int32_t *owner,
                            int32_t *slot, int32_t *members, void *stream);
BDM_API int64_t bdm_dispatch_owned_workspace_bytes(int64_t batch, int64_t time, int kw, int kr, int64_t local_banks);
BDM_API int bdm_dispatch_owned(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time, int kw,
                               int kr, int64_t bank_count, const int32_t *owner, const int32_t *slot, int rank,
                               int64_t local_banks, int64_t *order, int64_t *cu_seqlens, int64_t *inverse,
                               int64_t *tokens, int32_t *error_word, void *workspace, int64_t workspace_bytes,
                               void *stream);
BDM_API int bdm_combine_partial(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                const int32_t *owner, int64_t bank_count, int rank, int dtype, float *out,
                                void *stream);
BDM_API int bdm_norm_gate_f32(const float *combined, int64_t ntok, int64_t width, const void *gate, int64_t ld_gate,
                              const void *norm_weight, const void *norm_bias, float eps, int norm_mode, int dtype,
                              void *out, void *stream);

/*
 * One decode token per batch row.  Replaces inference.step's bank kernels
 * _decode_write, _decode_read and _decode_sum (inference.py:21-67,175-193).
 *   controls q,k,b,g [batch, H, S], v,w [batch, V]; routes [batch, kw|kr]
 *   state [batch, J, H, S, dv] (state_dtype) updated in place: every write
 *   bank of a row is rewritten in state_dtype, then reads (scale * M^T dtype(q*r),
 *   rounded to dtype) see the updated banks and are summed in ascending bank
 *   order with a rounding after each add into raw [batch, V] (dtype; may be NULL when
 *   gate is given).
 * With gate != NULL the step also applies the output interface's norm and gate to
 * the summed row, exactly as bdm_combine_norm_gate does for an already combined
 * input: out [batch, V] (dtype) = dtype(norm(raw) * dtype(sigmoid(gate))), gate
 * [batch, ld_gate] (dtype), norm_mode 1 = LayerNorm(norm_weight, norm_bias, eps),
 * 0 = RMS(norm_weight, eps).
 */
BDM_API int bdm_decode_step(const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                    const int64_t *write_idx, const void *write_w, const int64_t *read_idx, const void *read_w,
                    int64_t batch, int64_t bank_count, int heads, int bank_size, int head_value_width, int kw, int kr,
                    int dtype, int routed_decay, float scale, void *state, int state_dtype, void *raw,
                    const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias, float eps,
                    int norm_mode, void *out, void *stream);

/*
 * One whole decode step from the fused input projection, in one launch: the controllers
 * (_parameters.py:189-220, f_proj.1 computed in-kernel), both product-key routers
 * (gdn2_banks.py:74-114) and the bank step with the ordered read sum, norm and gate (as
 * bdm_decode_step, inference.py:161-194).  The step is then the projection GEMM, this call and
 * o_proj.  Results equal bdm_controllers + bdm_route_pair + bdm_decode_step bit for bit.
 *   proj [batch, ld] (dtype): one token per row; the column offsets name its q, k, v, f1
 *   (f1_width), b, w, read and write router logits (j1 + j2 each) and output-gate blocks.
 *   wf2 [H*S, f1_width] (dtype): f_proj.1's weight.  a_log [H], dt_bias [H*S] float.
 *   qk_norm 1 = 'nvidia', 0 = 'original'.  selected: banks per role (j1 * j2 == bank_count).
 *   state [batch, J, H, S, dv] (state_dtype) is updated in place.
 *   out [batch, H*dv] (dtype): the normalised and gated read sum, o_proj's input.
 */
BDM_API int bdm_decode_token_step(const void *proj, int64_t batch, int64_t ld, int64_t col_q, int64_t col_k,
                                  int64_t col_v, int64_t col_f1, int64_t col_b, int64_t col_w, int64_t col_read,
                                  int64_t col_write, int64_t col_gate, const void *wf2, int f1_width,
                                  const float *a_log, const float *dt_bias, int qk_norm, int j1, int j2,
                                  int selected, int64_t bank_count, int heads, int bank_size, int head_value_width,
                                  int dtype, int routed_decay, float scale, void *state, int state_dtype,
                                  const void *norm_weight, const void *norm_bias, float eps, int norm_mode,
                                  void *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BDM_B200_H */
