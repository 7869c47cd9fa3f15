/* fnx_b200.h -- C ABI of libfnx_b200.so, the B200 (sm_100a) W4A16 MoE expert path.
 *
 * Conventions (same as the reference's ctypes-loaded AscendC shims):
 *   - pointers are raw device pointers; `stream` is a cudaStream_t passed as void*;
 *   - every call launches asynchronously on `stream`, allocates nothing, never
 *     synchronises, and is capturable in a CUDA graph;
 *   - return 0 when launched, a negative code when an argument is rejected:
 *       -1 argument out of range, -2 unsupported shape, -3 alignment,
 *       -4 CUDA launch error, -5 workspace too small;
 *   - errors found on the device (a bounded wait that expired, an expert id outside
 *     [0, E)) are recorded in a device word read by fnx_device_errors().
 * Citations are to files of the reference tree (xyzhou613-dev/qwen-ascend).
 */
#ifndef FNX_B200_H
#define FNX_B200_H
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible exports (same symbol, argument order and meaning) ---- */

/* replaces kernels/expert_gather/gather.cpp:24 (fnx/expert_gather.py:22-28).
 * w int32 [E,K,N/8], s bf16 [E,G,N], ids int64 [10] -> ow int32 [K,10*N/8], os bf16 [G,10*N].
 * Accepts any N % 8 == 0 (the reference: N in {1280, 2560}); ids are not range-checked. */
int fnx_gather_pair(void* w, void* s, void* ids, void* ow, void* os, int K, int G, int N, void* stream);

/* replaces kernels/moe_epilogue/epilogue.cpp:41 (fnx/moe_epilogue.py:15-19): G=10, W=2560.
 * y bf16 [10, 10*2560] Cartesian down output, w bf16 [1,10], shared bf16 [1,2560], gate bf16 [1]. */
int fnx_moe_epilogue(void* y, void* w, void* shared, void* gate, void* out, void* stream);

/* replaces kernels/reduce/reduce.cpp:62 (fnx/weighted_reduce.py:33-39).
 * mode 1: out[t] = bf16(sum_g fp32(bf16(in[t*groups+g] * w[t*groups+g]))), w fp32 [batch,groups];
 * mode 2: rows via inverse int64 [batch*groups]; mode 0: mean of `groups` rows with bf16
 * elementwise weights [batch*groups, width].  order must be 0.  Any width >= 1, groups <= 64. */
int fnx_weighted_reduce(void* input, void* weights, void* inverse, void* output, int batch, int groups, int width,
                        int row_stride, int mode, int order, void* stream);

/* replaces kernels/post_ops/post_ops.cpp:91 (fnx/post_ops.py:14,39): width 2560,
 * out = bf16(e + bf16(s * bf16(sigmoid(g[t])))). */
int fnx_moe_merge(void* e, void* s, void* g, void* y, int batch, void* stream);

/* replaces libfnxw4gemv.so's fnx_w4gemv_launch as bound by fnx/w4gemv_op.py:42-43,153-158.
 * p4 [E,N,K/2] bytes (lay 1: lo=W[2j], hi=W[2j+1], x split xe/xo; lay 2: v2 layout, xe=xo=x),
 * s4t fp16 [E,K/32,N], ids int32 [nExp] (or NULL = slot order), y fp32 [nExp,N].
 * dbg and nblk are accepted and unused. */
int fnx_w4gemv_launch(void* p4, void* s4t, void* xe, void* xo, void* y, void* dbg, void* ids, int N, int K, int nExp,
                      int nblk, int lay, void* stream);

/* replaces fnx_w4gemv_launch_layers as bound by fnx/w4gemv_op.py:189-192: nL <= 64 layers in
 * one launch, host arrays of device pointers, x natural [nExp,K] fp32, ids = slot order. */
int fnx_w4gemv_launch_layers(void** p4, void** s4t, void** x, void** y, int nL, int N, int K, int nExp, int nblk,
                             int lay, void* dbg, void* stream);

/* replaces kernels/inject/inject.cpp:26 (fnx/native_inject.py:9-28): H = 2560, HC = 4.
 * out[t, b*H + c] = bf16(h[t, b*H + c] + bf16(y[t, c] * g[t, b])), h/out bf16 [batch, HC*H],
 * y bf16 [batch, H], g bf16 [batch, HC]. */
int fnx_inject(void* h, void* y, void* g, void* out, int batch, void* stream);

/* replaces kernels/post_ops/post_ops.cpp:25 (fnx/post_ops.py:22-26): the hyper-connection
 * activation of gated_residual (fnx/engine.py:832-851).  x bf16 [batch, 324] (320 mix + 4
 * inject columns) -> m = bf16(silu(bf16(x/4))) [batch, 320], g = bf16(2*bf16(sigmoid(bf16(x/4))))
 * [batch, 4].  mode bit 0: sigmoid as a rounded reciprocal; bit 1: silu as v * sigmoid. */
int fnx_hc_activation(void* x, void* m, void* g, int batch, int mode, void* stream);

/* replaces kernels/post_ops/post_ops.cpp:50 (fnx/post_ops.py:27-30): the branch mix of
 * gated_residual (fnx/engine.py:838-845).  x (hn), l (logits) bf16 [batch, 4*2560] ->
 * y bf16 [batch, 2560] = bf16(sum_b bf16(bf16(sigmoid(l_b)) * x_b) / 4). */
int fnx_hc_sigmoid_reduce(void* x, void* l, void* y, int batch, void* stream);

/* ---- widened forms of the reference kernels (shapes the AscendC kernels hard-code) ---- */

/* fnx_hc_activation with n_mix low-rank and HC inject columns. */
int fnx_hc_activation_ex(void* x, void* m, void* g, int batch, int n_mix, int HC, int mode, void* stream);
/* fnx_hc_sigmoid_reduce for any H and HC branches. */
int fnx_hc_sigmoid_reduce_ex(void* x, void* l, void* y, int batch, int H, int HC, void* stream);
/* rms_norm(x, w, gs=H) of fnx/engine.py:156-190 on hyper-connection rows: x, out bf16
 * [batch, HC*H]; every group of H normalised in fp32, times (1 + w) (w bf16 [HC*H]). */
int fnx_hc_rms_norm(void* x, void* w, void* out, int batch, int H, int HC, float eps, void* stream);

/* fnx_inject for any H % 8 == 0 and HC <= 64. */
int fnx_inject_ex(void* h, void* y, void* g, void* out, int batch, int H, int HC, void* stream);

/* fnx_gather_pair with any slot count; ids outside [0,E) copy zeros and set device error 2
 * (E <= 0 disables the check). */
int fnx_gather_pair_ex(void* w, void* s, void* ids, void* ow, void* os, int E, int K, int G, int N, int nslots,
                       void* stream);
/* fnx_moe_epilogue for y [k, k*width], w [1,k]. */
int fnx_moe_epilogue_ex(void* y, void* w, void* shared, void* gate, void* out, int k, int width, void* stream);
/* fnx_moe_merge for any width. */
int fnx_moe_merge_ex(void* e, void* s, void* g, void* y, int batch, int width, void* stream);

/* ---- the B200 MoE path (no single reference counterpart; each restates reference code) ---- */

/* Routing of fnx/engine.py:1811-1813: softmax(fp32(logits [T, ld] bf16, first E columns)
 * + bias fp32 [E] or NULL), top-k with ties to the lower expert id, w = bf16(p / sum p).
 * Outputs w_out bf16 [T,k], idx_out int64 [T,k], wf_out fp32 [T,k] (each may be NULL). */
int fnx_router_topk(void* logits, long long ld, void* bias, void* w_out, void* idx_out, void* wf_out, int T, int E,
                    int k, void* stream);

/* Expert-major permutation of fnx/engine.py:1817-1840, stable: idx int64 [n] ->
 * order int64 [n], inverse int64 [n], ends int64 [E] (cumulative counts), counts int64 [E]
 * (may be NULL).  workspace: fnx_moe_permute_workspace(n, E) bytes.  E <= 4096. */
size_t fnx_moe_permute_workspace(int n, int E);
int fnx_moe_permute(void* idx, void* order, void* inverse, void* ends, void* counts, int n, int E, void* workspace,
                    size_t ws_bytes, void* stream);

/* Expert-parallel dispatch layout (no counterpart in the reference, whose MoE runs on one
 * device; the exchange it serves is the NCCL all-to-all of the expert-parallel layer):
 * experts are owned in contiguous blocks of E/G by G ranks.  A stable counting sort of the
 * n = T*k slot ids by owner rank id / (E/G): order int64 [n] lists the slots owner-major
 * ((token*k + slot) order inside an owner), inverse int64 [n] is its inverse permutation
 * (the row of slot q in the owner-major buffer), counts int64 [G] the slots per owner.
 * E % G == 0; ids outside [0, E) set device error 2 and get no row.
 * workspace: fnx_ep_layout_workspace(n, G) bytes. */
size_t fnx_ep_layout_workspace(int n, int G);
int fnx_ep_dispatch_layout(const void* idx, int n, int E, int G, void* order, void* inverse, void* counts,
                           void* workspace, size_t ws_bytes, void* stream);

/* Row gather of the expert-parallel exchange: dst[p] = src[index[p] / index_div] for p < n,
 * bf16 rows of H elements with leading dimensions ld_src / ld_dst (index NULL: row p).
 * With ids_out (int64 [n]), also ids_out[p] = ids[index[p]] % ids_mod, the owner-local
 * expert id of a dispatched slot.  A source row outside [0, src_rows) writes zeros, sets
 * ids_out[p] = -1 and device error 2.  Dispatch: src = tokens, index = the owner-major
 * order of fnx_ep_dispatch_layout, index_div = k, ids = the routed ids, ids_mod = E/G.
 * Return: src = the owner's expert-major down output, index = the inverse of its local
 * expert permutation, index_div = 1. */
int fnx_ep_gather_rows(const void* src, long long ld_src, long long src_rows, const void* index, int index_div,
                       const void* ids, int ids_mod, void* dst, long long ld_dst, void* ids_out, long long n, int H,
                       void* stream);

/* Peer-memory exchange of the expert-parallel layer (the NVLink replacement of the
 * all-to-all; no counterpart in the reference).  Each of the G ranks (G <= 8, one node)
 * allocates one region of fnx_ep_p2p_region_bytes(G, H, k, T_cap) bytes with
 * fnx_ep_p2p_alloc (zero-filled), exports it with fnx_ep_p2p_export (a 64-byte CUDA IPC
 * handle) and imports every peer's with fnx_ep_p2p_import; fnx_ep_p2p_desc then fills an
 * opaque descriptor of fnx_ep_p2p_desc_bytes() bytes (host memory) from the G base pointers
 * (bases[rank] = its own).  T_cap: most tokens a rank brings to one call; Eg = E/G experts
 * per rank.  Capacities: cap = G*T_cap*k received slots, cap_tok = G*T_cap received token
 * rows (fnx_ep_p2p_capacity 0 / 1).
 * One layer call, on each rank's stream (every rank calls, in the same order), after
 * fnx_ep_dispatch_layout(idx) -> order, inverse, counts:
 *   fnx_ep_p2p_dedup(desc, order, counts, T, tok_index, tcounts)
 *       tok_index int32 [T*k]: each slot's token row among the rows sent (a token goes once
 *       to each owner holding any of its experts); tcounts int64 [G]: token rows per owner;
 *   fnx_ep_p2p_counts(desc, counts, tcounts)   exchanges the counts, starts the call's epoch;
 *   fnx_ep_p2p_push(desc, x, T, order, idx, tok_index)
 *       token rows and per-slot entries (owner-local expert, token row) to their owners, this
 *       rank's own tokens to its own region (the shared expert's rows);
 *   fnx_ep_p2p_wait(desc, 1)                  until every rank's rows for this rank landed;
 *   fnx_ep_p2p_recv_layout(desc, T, order_x, ends_x, pos, rows, sh_out, ws, ws_bytes)
 *       the owner's expert-major rows: expert 0 = the shared expert over its own T tokens,
 *       experts 1..Eg the received slots; order_x int64 [T + cap] (token rows of
 *       fnx_ep_p2p_local(desc, 0)), ends_x int64 [Eg + 1], pos int64 [cap] (each received
 *       slot's row), rows (pointers) [T + cap]: where each down row goes -- the shared rows
 *       to sh_out bf16 [T, H], each received slot's to its source's return buffer;
 *   grouped gate/up (fnx_moe_grouped_w4, epilogue 4, M = T + cap) and down
 *       (fnx_moe_grouped_w4_rows with out_rows = rows: the return happens in its epilogue);
 *   fnx_ep_p2p_signal(desc, 2)                the down rows are out;
 *   fnx_ep_p2p_wait(desc, 2)                  until this rank's rows are all back in
 *       fnx_ep_p2p_local(desc, 2) (bf16 [T_cap*k, H], owner-major: row inverse[q] is slot q).
 * Waits are bounded (device error 1 when a peer never arrives); a count beyond a capacity
 * sets device error 4 and its rows are dropped.  The setup and teardown calls (alloc, free,
 * export, import, close) and fnx_ep_p2p_received allocate or synchronise; the per-call ones
 * follow the conventions at the top of this file. */
size_t fnx_ep_p2p_region_bytes(int world, int H, int k, int T_cap);
int fnx_ep_p2p_alloc(size_t bytes, void** ptr);
int fnx_ep_p2p_free(void* ptr);
int fnx_ep_p2p_export(void* ptr, void* handle);
int fnx_ep_p2p_import(const void* handle, void** ptr);
int fnx_ep_p2p_close(void* ptr);
size_t fnx_ep_p2p_desc_bytes(void);
int fnx_ep_p2p_desc(void* desc, int rank, int world, void* const* bases, int H, int k, int T_cap, int Eg);
/* this rank's buffers: 0 recv_x bf16 [cap_tok + T_cap, H], 1 recv_e int64 [cap],
 * 2 yb bf16 [T_cap*k, H], 3 plan int64 (plan[0] = slots received this call), 4 recv_row int64 [cap] */
void* fnx_ep_p2p_local(const void* desc, int which);
long long fnx_ep_p2p_capacity(const void* desc, int which);
/* slots this rank received in its last call (synchronises with the device; for statistics) */
long long fnx_ep_p2p_received(const void* desc);
int fnx_ep_p2p_dedup(const void* desc, const void* order, const void* counts, int T, void* tok_index, void* tcounts,
                     void* stream);
int fnx_ep_p2p_counts(const void* desc, const void* counts, const void* tcounts, void* stream);
int fnx_ep_p2p_push(const void* desc, const void* x, int T, const void* order, const void* idx, const void* tok_index,
                    void* stream);
/* fnx_ep_p2p_push with flags (bit 0: do not copy the rank's own T token rows to its region's
 * shared-expert rows, for a caller that runs the shared expert from x itself) and a cap on the
 * launch's blocks (0: the default), so that a GEMM on another stream keeps its SMs. */
int fnx_ep_p2p_push_ex(const void* desc, const void* x, int T, const void* order, const void* idx,
                       const void* tok_index, int flags, int max_blocks, void* stream);
int fnx_ep_p2p_wait(const void* desc, int phase, void* stream);
int fnx_ep_p2p_signal(const void* desc, int phase, void* stream);
size_t fnx_ep_p2p_recv_workspace(const void* desc);
int fnx_ep_p2p_recv_layout(const void* desc, int T, void* order_x, void* ends_x, void* pos, void* rows, void* sh_out,
                           void* workspace, size_t ws_bytes, void* stream);
/* The received slots alone (no shared-expert rows): order_r [cap] the region row of each slot in
 * expert-major order, ends_r [Eg] cumulative from 0, pos [cap] each slot's position, rows_r [cap]
 * each position's down-row destination in its source's return buffer (the sink past the count). */
int fnx_ep_p2p_recv_layout_routed(const void* desc, void* order_r, void* ends_r, void* pos, void* rows_r,
                                  void* workspace, size_t ws_bytes, void* stream);

/* The LQP artifact's experts as the int4pack artifact, on the GPU (tools/repack_w4a16.py:41-70,
 * which needs CANN's npu_convert_weight_to_int4pack): v2o uint8 [E, N, K/2] offset-binary
 * (byte 64s+j of a row: low nibble W[128s+j] + 8, high nibble W[128s+64+j] + 8) -> w4 int32
 * [K, E, N/8] (expert_major = 0, the artifact's layout) or [E, K, N/8] (tools/repack_w4_em.py),
 * nibble t of word j = W[8j+t] two's complement.  N % 8 == 0, K % 128 == 0.  Byte-exact. */
int fnx_repack_v2o(const void* v2o, int E, int N, int K, int expert_major, void* w4, void* stream);

/* Load-time repack of the int4pack artifact (w4 int32 [E,K,Nw/8] expert-major, scales bf16
 * [E,K/gs,Nw]; tools/repack_w4a16.py, tools/repack_w4_em.py) into the tile blocks the B200
 * kernels stream: tiles int32 [E, Nw/128, K/64, 1088], one 4352-byte block per (expert,
 * feature tile m, k-block kb), contiguous along kb.  Word c*128 + (r ^ 8*(c%4)) (c < 8) holds the 8
 * weights k = 64kb+8c..+7 of tile row r as offset-binary nibbles in the order 0,2,4,6,1,3,5,7; bf16
 * 2048 + r (words 1024..1087) is row r's scale for the group holding kb (repeated in each
 * k-block of a group).  swiglu=1 orders tile rows as gate/up pairs (row 2i: gate feature
 * 64m+i, row 2i+1: up feature Nw/2+64m+i); swiglu=0: row r = 128m+r.
 * K % 64 == 0, Nw % 128 == 0, gs % 64 == 0, K % gs == 0.  (The reference's equivalent step is
 * the load-time scale cache of fnx/engine.py:653-659 and W4GemvOp.prepare_layer.) */
size_t fnx_w4_tiles_bytes(int E, int K, int Nw);
int fnx_repack_w4_tiles(const void* w4, const void* scales, void* tiles, int E, int K, int Nw, int gs, int swiglu,
                        void* stream);

/* Expert-major grouped W4A16 GEMM on tcgen05 (restated npu_grouped_matmul,
 * fnx/engine.py:723-753): rows [ends[e-1], ends[e]) use expert e.  Row r reads act row
 * row_index[r] / index_div (row_index NULL: act row r); a row index outside [0, act_rows)
 * reads zeros and sets device error 2.  tiles are the blocks of fnx_repack_w4_tiles
 * (swiglu=1 for epilogues 1 and 2); ends NULL means one group of M rows.
 * epilogue 0: out bf16 [M, Nw];  1: SwiGLU of gate = features [0,Nw/2), up = [Nw/2,Nw)
 * in fp32 on bf16-rounded inputs -> out [M, Nw/2];  2: the shared expert's SwiGLU
 * bf16(bf16(silu(g)) * u);  3: epilogue 1 for experts 0..E-2 and epilogue 2 for expert E-1
 * (the shared expert appended to the routed experts, run in the same launch);  4: the same
 * with the shared expert first (expert 0, epilogue 2) and the routed experts 1..E-1.
 * K % 64 == 0, Nw % 128 == 0. */
int fnx_moe_grouped_w4(const void* act, long long ld_act, long long act_rows, const void* row_index, int index_div,
                       const void* tiles, const void* ends, void* out, long long ld_out, int E, int M, int K, int Nw,
                       int epilogue, void* stream);
/* fnx_moe_grouped_w4 on at most max_ctas CTAs (0: all that fit; the CTA-pair kernel rounds down to
 * whole pairs), leaving SMs to kernels of another stream. */
int fnx_moe_grouped_w4_lim(const void* act, long long ld_act, long long act_rows, const void* row_index,
                           int index_div, const void* tiles, const void* ends, void* out, long long ld_out, int E,
                           int M, int K, int Nw, int epilogue, int max_ctas, void* stream);

/* fnx_moe_grouped_w4 with epilogue 0 whose output row r goes to out_rows[r] (a device array of
 * 16-byte aligned row pointers, bf16 [Nw] each, which may point into peers' memory): the
 * expert-parallel down projection writing each slot's row straight into its source's return
 * buffer. */
int fnx_moe_grouped_w4_rows(const void* act, long long ld_act, long long act_rows, const void* row_index,
                            int index_div, const void* tiles, const void* ends, void* out_rows, int E, int M, int K,
                            int Nw, void* stream);

/* fnx_moe_grouped_w4 (epilogues 0-2) over a selection of experts read in place, for ExpW4.apply /
 * apply_diag (fnx/engine.py:691-721, where the selected experts' weights are first gathered,
 * concatenated or index_select-ed into a copy): group e multiplies the tile blocks of expert
 * expert_ids[e] (int64 [E]) of the E_w experts in `tiles`; an id outside [0, E_w) reads expert 0
 * and sets device error 2. */
int fnx_moe_grouped_w4_sel(const void* act, long long ld_act, long long act_rows, const void* row_index,
                           int index_div, const void* tiles, int E_w, const void* expert_ids, const void* ends,
                           void* out, long long ld_out, int E, int M, int K, int Nw, int epilogue, void* stream);

/* W4GemvOp.weighted_sum (fnx/w4gemv_op.py:252-264): out fp32 [N] = sum over e of w[e] * y[e, :],
 * y fp32 [nE, N], w fp32 [nE] on the device; products rounded, summed in expert order. */
int fnx_weighted_sum_f32(const void* y, const void* w, void* out, int nE, int N, void* stream);

/* DenseW8.__call__ (fnx/engine.py:350-365): y bf16 [M,N] = x bf16 [M,K] . bf16(w8t int8 [K,N]
 * * sc bf16 [G,N]) with fp32 accumulation.  K % 64 == 0, N % 128 == 0. */
int fnx_w8a16_gemm(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int G, void* stream);

/* fnx_w8a16_gemm with a caller workspace: where one token tile leaves the GEMM too few tiles for
 * the SMs (M from 9 to about 128), K is split and the fp32 partials [s, M, N] go to ws, then are
 * summed in split order (deterministic); M <= 8 stays on the weight-streaming GEMV.  ws:
 * 16-byte aligned, at least fnx_w8a16_gemm_workspace(M, K, N, G) bytes (0: no split for this
 * shape; ws may be NULL). */
size_t fnx_w8a16_gemm_workspace(int M, int K, int N, int G);
int fnx_w8a16_gemm_ws(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int G, void* ws,
                      size_t ws_bytes, void* stream);

/* bf16 GEMM y [M, N] = x [M, K] . w [N, K]^T with fp32 accumulation (the router / concatenated
 * shared GEMM, fnx/engine.py:1787; the hyper-connection mix's GEMMs, fnx/engine.py:818-857):
 * both operands by TMA into a tcgen05 pipeline.  K % 64 == 0, ld_x % 8 == 0, x and w 16-byte
 * aligned; any N (the last feature tile is partial). */
int fnx_bf16_gemm_nt(const void* x, long long ld_x, const void* w, void* y, long long ld_y, int M, int K, int N,
                     void* stream);

/* Slot-order weighted reduce of the expert-major down output fused with the sigmoid-gated
 * shared merge (fnx/engine.py:1844-1853): yd bf16 [T*k, H], wf fp32 [T,k], inverse int64
 * [T*k] (or NULL), sh bf16 [T,H], gate bf16 at gate[t * gate_ld] -> out bf16 [T,H]. */
int fnx_moe_combine(void* yd, void* wf, void* inverse, void* sh, void* gate, long long gate_ld, void* out, int T, int k,
                    int H, void* stream);

/* fnx_moe_combine followed by the residual inject of the layer (fnx/engine.py:1945-1946:
 * `y = _moe(mixed); return inject(h, inj, y)`) in the same pass: out_hyper [T, HC*H] =
 * inject(hyper, inj, y) with y the combined output (also stored to `out` unless it is NULL).
 * k <= 16, H % 8 == 0, HC <= 64. */
int fnx_moe_combine_inject(void* yd, void* wf, void* inverse, void* sh, void* gate, long long gate_ld, void* hyper,
                           void* inj, void* out_hyper, void* out, int T, int k, int H, int HC, void* stream);

/* Whole decode MoE layer for M <= 16 tokens (fnx/engine.py:1786-1889 decode branch):
 * router bf16 [E+1, H] (row E = shared-expert gate), routed and shared experts as the
 * tile blocks of fnx_repack_w4_tiles (gate/up with swiglu=1, down with swiglu=0);
 * out bf16 [M,H], w_out bf16 [M,k], idx_out int64 [M,k] (may be NULL).
 * H % 256 == 0, I % 128 == 0, H, I <= 4096, E <= 512.
 * workspace: fnx_moe_decode_workspace(M,H,I,E,k) bytes, 16-byte aligned, zero-filled before
 * its first use and never cleared afterwards (its first word counts the calls made on it; the
 * values one call hands between CTAs carry that call's tag).  out 4-byte aligned.  Calls sharing
 * a workspace must not overlap on the GPU. */
size_t fnx_moe_decode_workspace(int M, int H, int I, int E, int k);
int fnx_moe_decode_w4(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                      const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H, int I,
                      int E, int k, void* workspace, size_t ws_bytes, void* stream);

/* The step before the decode layer with the router GEMV fused into it (fnx/engine.py:838-845, the
 * branch mix of gated_residual, then the router GEMV of fnx/engine.py:1786-1790 on its output):
 * y bf16 [M, H] = bf16(sum_b bf16(bf16(sigmoid(l_b)) * x_b) / HC) of x (hn) and l bf16 [M, HC*H],
 * and the router + shared-gate logits of y (router bf16 [E+1, H]) written into `workspace`, the
 * decode workspace of (M, H, I, E, k), tagged for the next decode launch on it.  Follow it with
 * fnx_moe_decode_w4_ex(..., flags = 1) on the same workspace and stream: that launch has no router
 * items and routes exactly as fnx_moe_decode_w4 would on y.  M <= 16, the decode shape rules. */
int fnx_hc_mix_router(const void* x, const void* l, void* y, const void* router, void* workspace, size_t ws_bytes,
                      int M, int H, int I, int E, int k, int HC, void* stream);
/* fnx_moe_decode_w4 with flags: bit 0, the router logits are already in the workspace
 * (fnx_hc_mix_router ran just before on it).  Without that call the launch records device error
 * bit 8 and ends at once, its outputs undefined. */
int fnx_moe_decode_w4_ex(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                         const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H,
                         int I, int E, int k, void* workspace, size_t ws_bytes, int flags, void* stream);

/* fnx_moe_decode_w4 for callers that cannot allocate device memory (no counterpart in the
 * reference): a plugin host or FFI binding that hands over only input and output buffers,
 * or a serving process that forbids device allocation after start-up.  The scratch is a
 * 4 MiB array compiled into the library (held by every GPU that loads it until exit); shapes
 * needing more than that (see fnx_moe_decode_workspace) return -5.  The first call on a
 * device looks the array's address up, so make it before any stream capture.  Every call on
 * a device shares the array, so calls that overlap on the GPU race.  Allocates nothing. */
int fnx_moe_decode_w4_noalloc(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                              const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H,
                              int I, int E, int k, void* stream);

/* ---- library ---- */
const char* fnx_b200_version(void);
/* device error bits since the last clear: 1 bounded wait expired, 2 expert id out of range,
 * 4 overflow, 8 a fnx_moe_decode_w4_ex(flags = 1) launch found no fresh router logits (no
 * fnx_hc_mix_router on its workspace since the last decode; its outputs are then undefined).
 * Synchronises with the device (cudaMemcpyFromSymbol). */
unsigned fnx_device_errors(int clear);

#ifdef __cplusplus
}
#endif
#endif
