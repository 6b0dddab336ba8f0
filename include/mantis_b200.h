/*
 * mantis_b200.h — C ABI of the B200-native MantisNet evaluator kernels.
 *
 * Every entry point takes caller-owned DEVICE pointers, sizes and a CUDA
 * stream (cudaStream_t passed as void*), launches asynchronously on that
 * stream, allocates nothing, and returns an mb_status. Host-side argument
 * validation happens before any launch; a failing check returns
 * MB_INVALID_ARGUMENT and mb_last_error() describes it. Index values are
 * validated inside the kernels: an out-of-range index skips the access and
 * records a code in the device error word, read with mb_device_error().
 *
 * dtype codes: MB_F32 = 0, MB_BF16 = 1. Index arrays are int64 (the
 * reference's torch.long) unless the name says i32. Row-major matrices take a
 * leading dimension `ld*` in elements.
 *
 * Each declaration names the reference interface it replaces, by path inside
 * the reference project (Cmiller132/Hexo-Shrimp-Bot).
 */
#ifndef MANTIS_B200_H
#define MANTIS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MB_OK = 0,
  MB_INVALID_ARGUMENT = 1,
  MB_LAUNCH_FAILED = 2,
  MB_TIMEOUT = 3,
  MB_UNSUPPORTED = 4,
  MB_DEVICE_ERROR = 5
} mb_status;

enum { MB_F32 = 0, MB_BF16 = 1 };

/* Library identity and diagnostics. */
int mb_version(void);
const char* mb_last_error(void);
/* Copies and optionally clears the device error word (synchronises `stream`). */
int mb_device_error(void* stream, uint32_t* code, int clear);

/* ---------------------------------------------------------------- tables --
 * Integer CSR derivations, bit-exact with the reference's torch.argsort(
 * stable=True) / torch.searchsorted(left) compositions.
 */

/* ptr[d] = first e with keys[e] >= d for d in [0, n_dest]; keys sorted,
 * in [0, n_dest). Replaces torch.searchsorted(sorted, arange(n+1)) at
 * python/mantisnet/mantisnet/cell_latents.py:146-160, cell_nodes.py:63-72,
 * window_latents.py:52-55. */
int mb_csr_from_sorted(const int64_t* keys, int64_t n, int64_t n_dest, int64_t* ptr, void* stream);

/* Stable argsort of non-negative int64 keys < 2^key_bits (LSD radix).
 * order[i] = index of the i-th smallest key, ties in input order; also writes
 * the sorted keys. Workspace size from mb_argsort_workspace. Replaces
 * torch.argsort(stable=True) at message_passing.py:511, cell_latents.py:133,148,
 * cell_nodes.py:60-70, window_latents.py:52. */
int mb_argsort_workspace(int64_t n, int key_bits, int64_t* bytes);
int mb_argsort(const int64_t* keys, int64_t n, int key_bits, int64_t* sorted_keys, int64_t* order,
               void* workspace, int64_t workspace_bytes, void* stream);

/* out[i] = src[idx[i]] for int64 arrays (index_select on the edge views). */
int mb_gather_i64(const int64_t* src, int64_t n_src, const int64_t* idx, int64_t n, int64_t* out, void* stream);

/* Radius class orbit + 48 * (own + 2 * on_axis), gathered through `order`
 * (order may be NULL for identity). model.py:867-869. */
int mb_radius_class(const int64_t* orbit, const int64_t* own, const int64_t* on_axis, const int64_t* order,
                    int64_t n, int64_t* out, void* stream);

/* window_pos[i] = window_slot[i] / max_w (model.py:919). */
int mb_div_i64(const int64_t* x, int64_t n, int64_t divisor, int64_t* out, void* stream);

/* ------------------------------------------------------- run reductions --
 * out[d, :] = sum_{e in [ptr[d], ptr[d+1])} values[gather[e], :]  (+ addend)
 * fp32 accumulation; `values` f32 or bf16, `out` f32 or bf16.
 * Optional addend: add[(add_idx ? add_idx[d] : d) * ld_add + col] (fp32).
 * Replaces mantisnet::aggregate_to_windows / aggregate_to_stones /
 * class_row_sum / incidence_row_sum (message_passing.py:191-227, 344-365;
 * kernel message_passing.py:40-99). */
int mb_run_reduce(const void* values, int values_dtype, int64_t ld_values, int64_t n_values,
                  const int64_t* gather, const int64_t* ptr, int64_t n_dest, int64_t width,
                  const float* add, int64_t ld_add, const int64_t* add_idx, int64_t n_add,
                  void* out, int out_dtype, int64_t ld_out, void* stream);

/* Action-row encoder: out[c] = sum_e relu(pre[win[e]] + table[cls[e]])
 *   + sum_o empty_counts[c, o] * relu(empty_base + table[empty_cls[o]]),
 * fp32 accumulation, run ptr over cells. Replaces mantisnet::action_row_encode
 * (row_encoder.py:368-380, 416-447) fused with the EMPTY-row term
 * (model.py:1049-1057). empty_counts may be NULL. Output row c starts at
 * out + c * ld_out (ld_out >= h, a multiple of the vector width). */
int mb_row_encode(const void* pre, int pre_dtype, int64_t n_pre, const float* table, int64_t n_table,
                  const int64_t* edge_window, const int64_t* edge_class, const int64_t* cell_ptr, int64_t n_cells,
                  const int64_t* empty_counts, const float* empty_base, const int64_t* empty_cls, int n_empty,
                  int64_t h, void* out, int out_dtype, int64_t ld_out, void* stream);

/* Relay cell pass (default config, §5.1b): pre[c] = sum x[w] + emb[cls];
 * val = relu(pre); out[w] = sum val over the window's cells. `scratch` holds
 * n_cov * h floats. Replaces mantisnet::cell_pass (relay.py:452-591). */
int mb_cell_pass(const void* x, int x_dtype, int64_t n_windows, const float* emb, int64_t n_cls,
                 const int64_t* cell_ptr, int64_t n_cov, const int64_t* edge_window, const int64_t* edge_class,
                 const int64_t* win_ptr, const int64_t* edge_wcell, int64_t h, float* scratch,
                 void* out, int out_dtype, void* stream);

/* The relay cell pass above without any allocation, for callers that cannot
 * allocate device memory (a host runtime that owns every device buffer, a
 * fixed memory budget): the (n_cov x h) scratch lives in a 16 MiB array
 * compiled into the library, so n_cov * h may not exceed 4,194,304; larger
 * calls return MB_INVALID_ARGUMENT. Each call outside a stream capture looks
 * up the array's address on its device (a call inside a capture reuses the
 * last one, so make the first call on a device before any capture). Calls
 * share the array: calls that overlap on the GPU race. This entry point has
 * no counterpart in the reference. */
int mb_cell_pass_noalloc(const void* x, int x_dtype, int64_t n_windows, const float* emb, int64_t n_cls,
                         const int64_t* cell_ptr, int64_t n_cov, const int64_t* edge_window, const int64_t* edge_class,
                         const int64_t* win_ptr, const int64_t* edge_wcell, int64_t h,
                         void* out, int out_dtype, void* stream);

/* ------------------------------------------------------------ attention --
 * Typed segment attention: per query row and head, online softmax over its
 * CSR run of sources; score = q.k / sqrt(hd) + bias[head, cls]; value =
 * v[src] (+ vcls[cls] when vcls != NULL; vcls f32 or bf16, (n_cls, heads * head_dim)).
 * Empty runs (or rows whose
 * skip_ptr run is non-empty) read zero with m = -inf, l = 0. m/l may be NULL.
 * Replaces mantisnet::cell_attention and mantisnet::cell_attention_plain
 * (cell_latents.py:834-940; kernel cell_latents.py:213-285). */
int mb_segment_attention(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                         int64_t n_q, int64_t n_src, int heads, int head_dim,
                         const float* bias, int64_t n_cls, const void* vcls, int vcls_dtype,
                         const int64_t* seg_ptr, const int64_t* src, const int64_t* cls, const int64_t* skip_ptr,
                         void* out, int out_dtype, int64_t ldo, float* m, float* l, void* stream);

/* The segment attention above for block-diagonal edge sets, with the same
 * result up to float rounding (m/l not produced): query rows and sources split into
 * n_groups groups (group g: rows [q_off[g], q_off[g+1]), sources
 * [s_off[g], s_off[g+1])) and every edge of a group-g row names a group-g
 * source; an edge outside its group is reported as an index error and
 * skipped. Each group's K/V columns are staged in shared memory once (groups
 * of more than stage_rows sources, or more than fit, read K/V from global
 * memory). q/k/v bf16 with 16-byte aligned rows; head_dim in {8, 16, 32, 64}
 * and heads * head_dim a multiple of 64; n_cls <= 2048 and the bias and
 * class value rows of one 64-column block must fit in shared memory. Replaces the radius
 * read mantisnet::cell_attention(q cells, k/v stones, radius tables)
 * (model.py:439-451, tables model.py:864-875; kernel cell_latents.py:213-285). */
int mb_segment_attention_grouped(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                                 int64_t n_q, int64_t n_src, int heads, int head_dim,
                                 const float* bias, int64_t n_cls, const void* vcls, int vcls_dtype,
                                 const int64_t* seg_ptr, const int64_t* src, const int64_t* cls,
                                 const int64_t* skip_ptr, const int64_t* q_off, const int64_t* s_off,
                                 int64_t n_groups, int64_t stage_rows, void* out, int out_dtype, int64_t ldo,
                                 void* stream);

/* The radius read (cells <- stones within distance 8) in two steps, for the
 * trunk's blocks to share the first (model.py:439-451 with the radius tables
 * of model.py:864-875; kernel cell_latents.py:213-285).
 * mb_radius_pack_edges: packed[e] = (src[e] - s_off[g]) << 11 | cls[e] for
 * every edge of group g's rows [q_off[g], q_off[g+1]) (edges [seg_ptr[q_off[g]],
 * seg_ptr[q_off[g+1]])), -1 (and a device error) where the stone is not one
 * of the group's [s_off[g], s_off[g+1]) or the class is not below n_cls
 * (n_cls <= 2048, fewer than 2^20 stones per group).
 * mb_radius_read: the result of mb_segment_attention_grouped on the packed
 * edges (head_dim 32, bf16 q/k/v and class rows, fp32 bias), rows of each
 * group visited in the order `order` gives (a permutation of the group's own
 * rows, NULL = ascending; the engine orders them by edge count). */
int mb_radius_pack_edges(const int64_t* src, const int64_t* cls, const int64_t* seg_ptr, const int64_t* q_off,
                         const int64_t* s_off, int64_t n_groups, int64_t n_q, int64_t n_edges, int64_t n_src,
                         int64_t n_cls, int32_t* packed, void* stream);
/* mb_radius_slots: the read order as a table of int32 quadruples (row, first
 * edge, edge count or 0 for a skipped row, 0) per slot, and the packed edges
 * (mb_radius_pack_edges) copied into slot order, each cell's run starting at
 * a multiple of four entries and padded with -1; both 16-byte aligned, the
 * copy mb_radius_slots_size entries long. Built once per forward; passed to
 * mb_radius_read as `slots` with the copy as `packed` (then `order`,
 * `seg_ptr` and `skip_ptr` are not read there). No counterpart in the
 * reference. */
int mb_radius_slots_size(int64_t n_q, int64_t n_groups, int64_t n_edges, int64_t* len);
int mb_radius_slots(const int32_t* packed, const int64_t* seg_ptr, const int64_t* skip_ptr, const int64_t* order,
                    const int64_t* q_off, int64_t n_groups, int64_t n_q, int64_t n_edges, int32_t* slots,
                    int32_t* packed_slots, int64_t packed_slots_len, void* stream);
int mb_radius_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int64_t n_q, int64_t n_src,
                   int heads, int head_dim, const float* bias, int64_t n_cls, const void* vcls,
                   const int64_t* seg_ptr, const int32_t* packed, const int64_t* skip_ptr, const int64_t* q_off,
                   const int64_t* s_off, const int64_t* order, const int32_t* slots, int64_t n_groups,
                   int64_t stage_rows, void* out, int out_dtype, int64_t ldo, void* stream);

/* Block-diagonal stone attention over [4 latents; stones] per position.
 * Padded mode (tok_off == NULL): q/k/v/out element (p, a, t, d) at
 * p*s_pos + a*s_head + t*s_row + d, keys t < seq_lens[p] live, query rows
 * past seq_lens[p] (up to t_pad) written as zeros — mantisnet::fused_attention
 * (attention.py:719-753, 892-904). Ragged mode: rows of position p are
 * [tok_off[p], tok_off[p+1]) with head stride s_head and row stride s_row;
 * only the first `max_queries` rows of each position are queries (4 = the
 * last block's latent-only read, model.py:647-669; -1 = all). In ragged mode
 * o_pos > 0 writes position p's rows at p*o_pos (a compact output), else at
 * the token rows themselves. Padded mode may also write lse (P, heads, t_pad)
 * fp32: m + log(l) of each query row's scaled scores, 0 for a padded row
 * (the auxiliary output of mantisnet::fused_attention, attention.py:155-162);
 * NULL skips it. */
int mb_stone_attention(const void* q, const void* k, const void* v, int dtype, int64_t n_pos, int heads, int head_dim,
                       int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* seq_lens, int64_t t_pad,
                       const int64_t* tok_off, int64_t max_tokens, int max_queries,
                       void* out, int out_dtype, int64_t o_pos, int64_t o_head, int64_t o_row, float* lse,
                       void* stream);

/* Engine of mb_stone_attention: 1 (the default) runs bf16 head_dim-32
 * calls with at most 320 keys per position on the tensor cores (S = Q K^T
 * and P V with tcgen05.mma, fp32 softmax, P rounded to bf16 for the second
 * product), 0 keeps every call on the CUDA-core kernel (fp32 P). Process-wide,
 * a measurement knob. No counterpart in the reference. */
int mb_stone_attention_engine(int tensor_cores);

/* Window-latent read: four latent queries per position attend over the
 * position's windows (order[offsets[p]..offsets[p+1]]). q (P, 4, H), k/v
 * (N_w, H), out (P, 4, H). m/l (P, 4, heads) may be NULL.
 * Replaces mantisnet::window_latent_read (window_latents.py:553-600). */
int mb_window_latent_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                          int64_t n_pos, int64_t n_windows, int heads, int head_dim, const int64_t* offsets,
                          const int64_t* order, void* out, int out_dtype, float* m, float* l, void* stream);

/* Window-latent broadcast: each window attends over its position's four
 * latent slots. q (N_w, H), k/v (P, 4, H), out (N_w, H).
 * Replaces mantisnet::window_latent_broadcast (window_latents.py:640-714). */
int mb_window_latent_broadcast(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                               int64_t n_pos, int64_t n_windows, int heads, int head_dim, const int64_t* window_pos,
                               void* out, int out_dtype, float* m, float* l, void* stream);

/* Dense 4x4 latent self-mix per position and head, fp32 softmax
 * (model.py:516-526). q/k/v/out (P, 4, H). */
int mb_latent_mix(const void* q, const void* k, const void* v, int64_t ld, int dtype, int64_t n_pos, int heads,
                  int head_dim, void* out, int out_dtype, void* stream);

/* -------------------------------------------------------------- backward --
 * Gradients for the fit path, deterministic (no atomics; every sum in a
 * fixed order), fp32 math and fp32 gradients on f32 or bf16 inputs. Scatters
 * are gathers over stable permutations the caller derives once (edges by
 * source / class / window: mb_argsort + mb_csr_from_sorted). Softmax
 * backward per row i: D_i = sum_j P_ij dP_ij, dS_ij = P_ij (dP_ij - D_i).
 */

/* Typed segment attention (mantisnet::cell_attention_backward and
 * cell_attention_plain_backward, cell_latents.py:869-990; kernels
 * cell_latents.py:287-543): from the forward's m, l (n_q, heads) and the
 * output gradient (n_q, heads * head_dim) fp32, writes dq, dk, dv (row
 * layouts of q and k), dbias (heads, n_cls) and, with vcls, dvcls (n_cls,
 * heads * head_dim). qid (E): each edge's query row; src_perm / src_ptr: the
 * edges by source (stable) and their CSR over sources; cls_perm / cls_ptr:
 * by class. alpha_ws and dscore_ws: (E, heads) fp32 workspaces. Width
 * heads * head_dim in {32, 64, 128, 256}. */
int mb_segment_attention_backward(const void* q, const void* k, const void* v, int dtype, int64_t n_q, int64_t n_src,
                                  int heads, int head_dim, const float* bias, int64_t n_cls, const void* vcls,
                                  int vcls_dtype, const int64_t* seg_ptr, const int64_t* src, const int64_t* cls,
                                  const int64_t* qid, const float* m, const float* l, const float* grad_out,
                                  int64_t n_edges, const int64_t* src_perm, const int64_t* src_ptr,
                                  const int64_t* cls_perm, const int64_t* cls_ptr, float* alpha_ws, float* dscore_ws,
                                  float* dq, float* dk, float* dv, float* dbias, float* dvcls, void* stream);

/* Stone attention (mantisnet::fused_attention_backward, attention.py:823-890;
 * kernels attention.py:229-531), padded (P, A, T, D) layout of the forward
 * with its lse (P, A, T): dq, dk, dv (P, A, T, D) contiguous fp32; rows at or
 * past seq_lens[p] get zero gradients. dsum_ws: (P, A, T) fp32 workspace. */
int mb_stone_attention_backward(const void* q, const void* k, const void* v, const void* out, const void* grad_out,
                                int dtype, int64_t n_pos, int heads, int head_dim, int64_t s_pos, int64_t s_head,
                                int64_t s_row, const int32_t* seq_lens, int64_t t_pad, const float* lse,
                                float* dsum_ws, float* dq, float* dk, float* dv, void* stream);

/* Window-latent read and broadcast (mantisnet::window_latent_read_backward /
 * window_latent_broadcast_backward, window_latents.py:589-700; kernels
 * window_latents.py:270-473), row layouts of the forward (read: q (P * 4,
 * H), k/v (N_w, H); broadcast: q (N_w, H), k/v (P * 4, H)) with its fp32
 * out (read only), m, l and output gradient; window_pos per window, the
 * position CSR offsets / order of mb_window_latent_read. Broadcast
 * workspaces p_ws, ds_ws: (N_w, 4, heads) fp32. */
int mb_window_latent_read_backward(const void* q, const void* k, const void* v, int dtype, const float* out,
                                   const float* m, const float* l, const float* grad_out, const int64_t* window_pos,
                                   const int64_t* offsets, const int64_t* order, int64_t n_pos, int64_t n_windows,
                                   int heads, int head_dim, float* dq, float* dk, float* dv, void* stream);
int mb_window_latent_broadcast_backward(const void* q, const void* k, const void* v, int dtype, const float* m,
                                        const float* l, const float* grad_out, const int64_t* window_pos,
                                        const int64_t* offsets, const int64_t* order, int64_t n_pos,
                                        int64_t n_windows, int heads, int head_dim, float* p_ws, float* ds_ws,
                                        float* dq, float* dk, float* dv, void* stream);

/* Action-row encoder (the backward of mantisnet::action_row_encode,
 * row_encoder.py:114-207, 386-413): out[c] = sum_e relu(pre[win_e] +
 * table[cls_e]) gives grad_pre (n_pre, h) and grad_table (n_table, h) fp32,
 * the output gradient (n_cells, h) fp32 where the pre-activation is
 * positive; win_perm / win_ptr and cls_perm / cls_ptr: the edges by window
 * and by class. h in {32, 64, 128, 256}. */
int mb_row_encode_backward(const void* pre, int pre_dtype, int64_t n_pre, const float* table, int64_t n_table,
                           const int64_t* edge_window, const int64_t* edge_class, const int64_t* edge_cell,
                           int64_t n_edges, const float* grad_out, int64_t n_cells, int64_t h,
                           const int64_t* win_perm, const int64_t* win_ptr, const int64_t* cls_perm,
                           const int64_t* cls_ptr, float* grad_pre, float* grad_table, void* stream);

/* ------------------------------------------------------- rows and norms -- */

/* LayerNorm over rows of width h (fp32 statistics, eps), input f32 or bf16,
 * optional row gather in_rows[i] (NULL = identity). torch.nn.LayerNorm as
 * used throughout model.py. */
int mb_layer_norm(const void* x, int x_dtype, int64_t ldx, const int64_t* in_rows, int64_t n, int64_t h,
                  const float* gamma, const float* beta, float eps, void* out, int out_dtype, int64_t ldo,
                  void* stream);

/* Residual update fused with the LayerNorms that read it next:
 *   x[r] += y[r] (+ y_bias)           (skipped when y == NULL)
 *   o_j[r] = LN(x[r]; g_j, b_j)        for each given output j (up to 3, in order)
 * x fp32 (in place), y f32/bf16, outputs f32/bf16 with their own strides.
 * Replaces the residual-add + nn.LayerNorm pairs between the trunk's stages
 * (model.py:436-452, 480-489, 539-541, 570-580, 681-692, 973-985). */
int mb_add_ln(float* x, int64_t ldx, const void* y, int y_dtype, int64_t ldy, const float* y_bias, int64_t n,
              int64_t h, float eps, const float* g0, const float* b0, void* o0, int o0_dtype, int64_t ld0,
              const float* g1, const float* b1, void* o1, int o1_dtype, int64_t ld1, const float* g2,
              const float* b2, void* o2, int o2_dtype, int64_t ld2, void* stream);

/* out[i] = ta[ia[i]] + (tb ? tb[ib ? ib[i] : i] : 0): embedding lookups and
 * their sums (model.py:909-912, 929). fp32 tables and output. */
int mb_embed(const float* ta, int64_t n_ta, const int64_t* ia, const float* tb, int64_t n_tb, const int64_t* ib,
             int64_t n, int64_t h, float* out, void* stream);

/* Initial cell state: covered cells (cov_ptr run non-empty) take
 * `covered_row` (+ optional per-cell addend rows), the rest take
 * nearest_table[cell_nearest]. model.py:926-935. */
int mb_cell_init(const int64_t* cov_ptr, const int64_t* cell_nearest, const float* nearest_table, int64_t n_nearest,
                 const float* covered_row, const float* covered_add, int64_t n_cells, int64_t h, float* out,
                 void* stream);

/* Residual update: x[row(i)] += y[i]; x and y each f32 or bf16 (row map may
 * be NULL). */
int mb_residual_add(void* x, int x_dtype, int64_t ldx, const int64_t* rows, const void* y, int y_dtype, int64_t ldy,
                    int64_t n, int64_t h, void* stream);

/* x[i] = act(x[i] + t[idx[i]]) with act = relu when relu != 0: the per-position
 * token half of the decoder MLP joined per legal cell (model.py:1091). */
int mb_add_gather(void* x, int x_dtype, int64_t ldx, const void* t, int t_dtype, int64_t ldt, int64_t n_t,
                  const int64_t* idx, int64_t n, int64_t h, int relu, void* stream);

/* Token layout for stone attention: tokens of position p are its 4 latent
 * rows then its stones. gather: tok = [g; s] per position; scatter-add:
 * g += tok_out[latent rows], s += tok_out[stone rows] (model.py:622-646). */
int mb_tokens_gather(const float* g, const float* s, const int64_t* stone_off, const int64_t* tok_off,
                     int64_t n_pos, int64_t h, float* tok, void* stream);
int mb_tokens_scatter_add(float* g, float* s, const int64_t* stone_off, const int64_t* tok_off, int64_t n_pos,
                          int64_t h, const void* tok_out, int dtype, int update_stones, void* stream);

/* Mean of ln(g) over the 4 latent rows: out (P, h) fp32 (model.py:973). */
int mb_latent_mean(const float* g_ln, int64_t n_pos, int64_t h, float* out, void* stream);

/* Value head (model.py:1160-1183): per position p the rows [g[p]; its
 * windows (win_order[win_off[p] .. win_off[p+1]), NULL order = identity)],
 * each LayerNorm'd with (ln_g, ln_b, eps), are read by nq <= 4 queries
 * (queries (nq, h) fp32) with one head of width h, scores scaled by
 * 1/sqrt(h) and slots (window_slot - p * max_w; 0 for g[p]) that value_valid
 * (n_pos, max_w) marks invalid left out; the nq read rows, concatenated,
 * go through relu(w1 x + b1) (w1 (vh, nq * h)) and w2 x + b2 (w2 (bins, vh))
 * to logits, whose softmax is dist and whose expectation over centers is
 * value. g (n_pos, h) fp32, w (n_windows, ldw) f32 or bf16; all fp32 math.
 * h in {32, 64, 128, 256, 512}, vh and bins <= 256. */
int mb_value_head(const float* g, const void* w, int w_dtype, int64_t ldw, int64_t n_windows, const int64_t* win_off,
                  const int64_t* win_order, const int64_t* window_slot, const uint8_t* value_valid, int64_t n_pos,
                  int64_t max_w, int64_t h, const float* ln_g, const float* ln_b, float eps, const float* queries,
                  int nq, const float* w1, const float* b1, int vh, const float* w2, const float* b2, int bins,
                  const float* centers, float* value, float* dist, float* logits, void* stream);

/* Q composition (model.py:177-220, segments.py:24-31): per cell
 * p = softmax(critic[c, 0:3]); q_values = p0 - p1;
 * q_score = q_values / max(max over the position's cells of (p0 + p1), floor). */
int mb_compose_q(const float* critic, int64_t ld_critic, const int64_t* offsets, int64_t n_pos, float mass_floor,
                 float* q_score, float* q_values, void* stream);

/* ------------------------------------------------------------- GEMM ------
 * out = act(A @ W^T + bias) (+ residual) for row-major A (M, K), W (N, K).
 * Replaces the nn.Linear calls of model.py (the reference runs them through
 * cuBLAS under autocast). */
int mb_linear(const void* a, int a_dtype, int64_t lda, int64_t m, int64_t k, const void* w, int w_dtype,
              const float* bias, int64_t n, int relu, void* out, int out_dtype, int64_t ldo, void* stream);

/* Fused row GEMM on tcgen05 tensor cores (sm_100a), K = N = 256 (see
 * mb_gemm_rows_ex for the other shapes):
 *   out[r] = act(LN(x[r]) @ W^T + bias)            (gamma != NULL: x fp32, LayerNorm prologue)
 *   out[r] = act(x[r] @ W^T + bias)                (gamma == NULL: x bf16)
 * with either a bf16 output (out, ldo) or an in-place fp32 residual update
 * residual[r] += result (exactly one of the two). W is passed as the image
 * produced by mb_gemm_weight_image (256 x 256 bf16 -> 128 KB swizzled).
 * Replaces the LayerNorm -> nn.Linear -> residual-add chains of the trunk
 * (model.py:425-489, 506-540, 570-580, 609-619). */
int mb_gemm_weight_image(const void* w, int64_t n, int64_t k, void* image, void* stream);
int mb_gemm_rows(const void* x, int x_dtype, int64_t ldx, int64_t m, const float* gamma, const float* beta, float eps,
                 const void* w_image, const float* bias, int relu, void* out, int64_t ldo, float* residual,
                 int64_t ldr, void* stream);

/* The row GEMM above for every projection shape of the model: K = 256 or
 * 512 (bf16 rows; the LayerNorm prologue takes K = 256), N any multiple of
 * 128 (a row tile's N blocks run back to back on the tile held in shared
 * memory), w_image = mb_gemm_weight_image of the (N, K) weight. With `out`
 * (bf16, ldo >= n) an optional fp32 addend `add` (ld_add) is summed before the
 * activation; `residual` (fp32, N = 256) takes the in-place update instead.
 * A bf16 `out` is written by tensor-map stores of 32 x 32 boxes, so m must be
 * below 2^31 with `out` too; MB_LAUNCH_FAILED if the driver's tensor-map
 * encoder cannot be had. Replaces every nn.Linear of the trunk and the decoder (model.py:246-260,
 * 425-692 Q / K|V / FFN / PairMlp projections, 1031-1139 decoder GEMMs),
 * which the reference runs through cuBLAS under autocast. */
int mb_gemm_rows_ex(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, const float* gamma,
                    const float* beta, float eps, const void* w_image, int64_t n, const float* bias, int relu,
                    const float* add, int64_t ld_add, void* out, int64_t ldo, float* residual, int64_t ldr,
                    void* stream);

/* Launch plan of the bf16-output row GEMMs (a measurement knob; the
 * defaults are the measured best): store_plan 0 streams W K-blocks per row
 * tile, 1 holds a whole N block of W in shared memory per CTA (256 columns
 * at K = 256, 128 columns at K = 512 when N <= 256);
 * ln_plan 0 stages the LayerNorm prologue's fp32 rows in 32-row groups, 1
 * weight-stationary with per-row loads, 2 per-row loads with W streamed.
 * Process-wide; not for use while launches are being issued from other
 * threads. No counterpart in the reference. */
int mb_gemm_set_plan(int store_plan, int ln_plan);

/* A decoder head's last two layers in one launch (the reference's _PairMlp
 * on a cell row and its position's row, model.py:246-260 called from
 * _cell_scores, model.py:1031-1139):
 *   out[r, j] = b_out[j] + sum_c w_out[j, c] * relu(x[r] W^T + bias + tok[tok_idx[r]])[c]
 * x (m, 256) bf16; W (N, 256), N = 128 or 256, as mb_gemm_weight_image;
 * tok (n_tok, N) bf16 rows (the position half, already projected);
 * tok_idx (m) int64 position of each row; w_out (n_out, N) fp32 row-major,
 * 1 <= n_out <= 4; out (m, n_out) fp32 with leading dim ldo. */
int mb_gemm_rows_head(const void* x, int64_t ldx, int64_t m, const void* w_image, int64_t n, const float* bias,
                      const void* tok, int64_t ld_tok, int64_t n_tok, const int64_t* tok_idx, const float* w_out,
                      const float* b_out, int n_out, float* out, int64_t ldo, void* stream);

/* Fused projection + residual update + LayerNorms on the tensor cores:
 *   x[r] += a[r] W^T + bias;  out_j[r] = LN_j(x[r])  for each given output j,
 * a (m, 256) bf16 rows, x = residual (m, 256) fp32 rows updated in place,
 * w_image from mb_gemm_weight_image; up to three LayerNorm outputs (gamma,
 * beta, destination, dtype, leading dim; fill in order, NULL to stop; dtype
 * must be MB_BF16), each from the same updated row with two-pass fp32
 * statistics. One pass over the
 * residual row replaces the reference's Linear, residual add and following
 * LayerNorm calls (model.py:397-490 cell stage, :543-692 window updates). */
int mb_gemm_rows_ln(const void* a, int64_t lda, int64_t m, const void* w_image, const float* bias, float* residual,
                    int64_t ldr, float eps, const float* g0, const float* b0, void* o0, int o0_dtype, int64_t ld0,
                    const float* g1, const float* b1, void* o1, int o1_dtype, int64_t ld1, const float* g2,
                    const float* b2, void* o2, int o2_dtype, int64_t ld2, void* stream);

/* ------------------------------------------------- isolated-op workloads --
 * The two isolated ops of the benchmark suite. Neither exists as an op in the
 * reference; each restates its workload definition, and the CPU restatements
 * in oracle/isolated.py pin them.
 */

/* Hex message passing over cell tokens, fused on the tensor cores:
 *   out[i] = x[i] + W mean_{s: nbr[i,s] >= 0} x[nbr[i,s]] + bias
 * x, out (n, 256) bf16 rows (leading dims ldx, ldo; out must not alias x);
 * nbr (n, 6) int32 rows of x in the reference adjacency slot order
 * (builder.py:458-471: axes Q, R, QR of builder.py:32, step -1 then +1), -1
 * where the neighbour is not a token; a row with no neighbour aggregates to
 * zero. w_image from mb_gemm_weight_image of W (256 x 256); bias fp32 (256,)
 * or NULL. The mean is rounded to bf16 before the product; fp32 accumulate. */
int mb_hex_message_pass(const void* x, int64_t ldx, int64_t n, const int32_t* nbr, const void* w_image,
                        const float* bias, void* out, int64_t ldo, void* stream);

/* Attention over a position's cell tokens with an additive per-head bias
 * indexed by the relative axial offset, on the tensor cores:
 *   out[p,h,i] = sum_j softmax_j(q_i.k_j / sqrt(32) + bias[dq+16, dr+16, h]) v_j
 * dq, dr = key coordinate minus query coordinate (axial q, r), each clamped
 * to [-16, 16]; keys j < valid[p] only; query rows i >= valid[p] are written
 * as zeros. q/k/v element (p, h, t, d) at p*s_pos + h*s_head + t*s_row + d,
 * out likewise with o_*; bf16, head_dim 32, length <= 256; coords (n_pos,
 * length, 2) int32; valid (n_pos,) int32; bias (33, 33, heads) fp32. The
 * score arithmetic follows the reference's additive-bias attention
 * (cell_latents.py:552-555 adds a gathered fp32 bias to fp32 scores). */
int mb_axial_attention(const void* q, const void* k, const void* v, int64_t n_pos, int heads, int head_dim,
                       int64_t length, int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* coords,
                       const int32_t* valid, const float* bias, void* out, int64_t o_pos, int64_t o_head,
                       int64_t o_row, void* stream);

/* ---------------------------------------------------------------- KLENT --
 * Policy improvement over each position's legal cells (reference
 * python/mantisnet/mantisnet/klent/improve.py:27-69, eq. 3 of the KLENT
 * note; Rust crates/models/mantisnet/src/improvement.rs:104): pi' = softmax(
 * (q_score + tau log softmax(logits)) / (tau + lam)) into probs, and per
 * position v_hat = E_pi'[q_values], kl = KL(pi' || pi), norm_entropy =
 * H(pi') / log|A| (0 for one legal cell). offsets: (n_pos + 1) int64 segment
 * bounds over n cells. With uniforms (n_pos float64 draws in [0, 1)) it also
 * draws each position's move as the self-play loop does
 * (klent/selfplay.py:180-190): stored = pi' renormalised in float64 (written
 * as float32), ranks = first cell whose cumulative probability reaches the
 * uniform (clipped to the segment), pi_top1 and pi_chosen in float64.
 * uniforms NULL skips the draw. All device pointers. */
int mb_klent_improve(const float* policy_logits, const float* q_score, const float* q_values, const int64_t* offsets,
                     int64_t n_pos, int64_t n, float tau, float lam, float* probs, float* v_hat, float* kl,
                     float* norm_entropy, const double* uniforms, float* stored, int64_t* ranks, double* pi_top1,
                     double* pi_chosen, void* stream);

/* ranks[p] = the index within segment p ([offsets[p], offsets[p+1]) of x)
 * of its largest value, the first one on ties (torch.argmax over the
 * segment), -1 for an empty segment: the Gumbel search's per-leaf move from
 * the improved policy (klent/search.py:246-249). Device pointers. */
int mb_segment_argmax(const float* x, const int64_t* offsets, int64_t n_pos, int64_t n, int64_t* ranks, void* stream);

/* --------------------------------------------------------------- encoder --
 * Host-side batch builder: game positions to the collated batch arrays that
 * the evaluator reads. HOST pointers, no stream, no GPU needed. Replaces the
 * reference's batch builder: the Python build / collate / batch_from_arrays
 * (python/mantisnet/mantisnet/builder.py:486-956 with the relay views of
 * relay.py:48-94) and the production Rust encoder
 * (crates/models/mantisnet/src/encoder.rs:1047-1660). Every array equals the
 * Python builder's, order included.
 *
 * Usage: mb_encode_positions builds every position's graph (threads: 0 = one
 * per hardware thread) and returns a handle; mb_encoding_sizes reports the
 * batch sizes; the caller allocates one buffer per field (host memory,
 * pinned or not) and mb_encoding_fill writes them; mb_encoding_free releases
 * the handle. A position the builder refuses (no legal moves, moves_remaining
 * not 1 or 2, duplicate stones, a legal cell occupied or beyond distance 8
 * of every stone) fails the whole call with MB_INVALID_ARGUMENT and a message
 * naming the position.
 *
 * Inputs: positions i in [0, n_pos) own stones [stone_off[i], stone_off[i+1])
 * of stone_qr (axial q, r pairs) and stone_owner, the player to move
 * mover[i], legal cells [legal_off[i], legal_off[i+1]) of legal_qr, and
 * moves_remaining[i] (1 or 2). */
typedef struct mb_encoding mb_encoding;

/* sizes[]: */
enum {
  MB_ENC_P = 0, MB_ENC_NS, MB_ENC_NW, MB_ENC_NINC, MB_ENC_NC, MB_ENC_NRADIUS, MB_ENC_NADJ, MB_ENC_NDEC,
  MB_ENC_MAX_T, MB_ENC_MAX_W, MB_ENC_NCOVERED, MB_ENC_NSIZES
};
/* fields[], each a host buffer: shape in sizes[] terms, dtype i64 unless
 * noted (u8 = one byte per flag, 0 or 1). */
enum {
  MB_ENC_STONE_OWN = 0,  /* (NS) */
  MB_ENC_WINDOW_FEAT,    /* (NW) */
  MB_ENC_WINDOW_ID,      /* (NW, 3): axis, start q, start r */
  MB_ENC_MOVES_IDX,      /* (P) */
  MB_ENC_INC_STONE,      /* (NINC) */
  MB_ENC_INC_WINDOW,     /* (NINC) */
  MB_ENC_INC_CLASS,      /* (NINC) */
  MB_ENC_STONE_SLOT,     /* (NS) */
  MB_ENC_COORDS,         /* (P, MAX_T, 2) i32 */
  MB_ENC_ATTN_VALID,     /* (P, MAX_T) u8 */
  MB_ENC_WINDOW_SLOT,    /* (NW) */
  MB_ENC_VALUE_VALID,    /* (P, MAX_W) u8 */
  MB_ENC_LEGAL_OFFSETS,  /* (P + 1) */
  MB_ENC_CELL_POS,       /* (NC) */
  MB_ENC_CELL_NEAREST,   /* (NC) */
  MB_ENC_RADIUS_SRC,     /* (NRADIUS) */
  MB_ENC_RADIUS_DST,
  MB_ENC_RADIUS_ORBIT,
  MB_ENC_RADIUS_OWN,
  MB_ENC_RADIUS_ON_AXIS,
  MB_ENC_ADJ_SRC,        /* (NADJ) */
  MB_ENC_ADJ_DST,
  MB_ENC_ADJ_AXIS,
  MB_ENC_DEC_CELL,       /* (NDEC) */
  MB_ENC_DEC_WINDOW,
  MB_ENC_DEC_CLASS,
  MB_ENC_RELAY_CELL_PTR, /* (NCOVERED + 1) */
  MB_ENC_RELAY_WINDOW,   /* (NDEC) */
  MB_ENC_RELAY_CLASS,    /* (NDEC) */
  MB_ENC_RELAY_WIN_PTR,  /* (NW + 1) */
  MB_ENC_RELAY_WCELL,    /* (NDEC) */
  MB_ENC_RELAY_CLS_PTR,  /* (727) */
  MB_ENC_RELAY_CCELL,    /* (NDEC) */
  MB_ENC_ACT_CLASS,      /* (NDEC) */
  MB_ENC_ACT_REV,        /* (NDEC) */
  MB_ENC_ACT_EMPTY,      /* (NC, 3) */
  MB_ENC_ACT_TACTICAL,   /* (NC, 11) f32 */
  MB_ENC_NFIELDS
};
int mb_encode_positions(int64_t n_pos, const int64_t* stone_off, const int64_t* stone_qr, const int64_t* stone_owner,
                        const int64_t* mover, const int64_t* legal_off, const int64_t* legal_qr,
                        const int64_t* moves_remaining, int threads, mb_encoding** out);
int mb_encoding_sizes(const mb_encoding* encoding, int64_t* sizes);
int mb_encoding_fill(const mb_encoding* encoding, void* const* fields, int threads);
/* The same arrays with every int64 field written as int32 (the narrow
 * layout: half the host memory and host-to-device bytes; the evaluator
 * widens them on the device). Refuses a batch whose sizes do not fit int32.
 * No counterpart in the reference. */
int mb_encoding_fill_narrow(const mb_encoding* encoding, void* const* fields, int threads);
int mb_encoding_free(mb_encoding* encoding);
/* The encoder's vocabulary tables (0 window-pattern rank [729], 1 occupied-
 * slot class [729 x 6], 2 decoder class [729 x 6], 3 post-placement class
 * [729 x 6], 4 displacement orbit [25 x 25]; -1 where undefined), for
 * checking them against another derivation. Follows the reference
 * definitions at builder.py:41-229. */
int mb_encoder_table(int which, int64_t* out, int64_t capacity);

#ifdef __cplusplus
}
#endif

#endif /* MANTIS_B200_H */
