/*
 * sparsefold_b200 — C ABI of the B200 (sm_100a) kernels for the AF3 trunk hot path.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, element
 * counts and a CUDA stream, returns an `int` status (SF_OK == 0), and never
 * throws.  On failure `sf_last_error()` returns a message for the calling
 * thread.  The caller allocates every input, output and workspace buffer; the
 * library calls no cudaMalloc or cudaFree.  Its only device state is two
 * file-scope `__device__` arrays that every GPU loading the library holds
 * until the process exits: a 4-byte status word per device (see
 * sf_device_status) and the fixed 16 MiB scratch array of
 * sf_transition_noalloc (see the notes at that entry point).  Their device
 * addresses are looked up once per device and cached; calls made after
 * cudaDeviceReset() on a device are not supported.  Work is enqueued
 * asynchronously on `stream`.
 *
 * Conventions
 *  - dtype (`SF_F32` / `SF_BF16`) is the element type of the activation
 *    tensors (pair z, single s, intermediate buffers).  Weights passed as
 *    `const void*` have the same dtype; LayerNorm scales/offsets and Linear
 *    biases are always fp32.  Arithmetic accumulates in fp32.
 *  - Weights are "out x in" matrices (`Wt[n_out][k_in]`, k contiguous), the
 *    transpose of the reference's `x @ W` layout; the Python `prepare()` step
 *    builds them.
 *  - Pair tensors are position-major `[rows][n][c]` (channels contiguous).
 *    Masks are `uint8_t` (0 / 1) per token.
 *  - `rows` is the number of pair rows this call owns (all `n` on one device,
 *    `n / P` on a row shard) and `row_offset` the global index of its first row.
 *
 * Reference interfaces replaced (paths in HenryRenYz/SparseFold src/sparsefold/):
 *  sf_attention            backends/torch/attention/sdpa.py:22-121  dot_product_attention
 *  sf_layernorm            model/layers/primitives.py:471-497       LayerNorm.forward
 *  sf_tri_mult_*           model/trunk/blocks.py:484-566            TriangleMultiplication.forward
 *  sf_tri_attention_*      model/trunk/blocks.py:270-366            GridSelfAttention.forward/_attention
 *  sf_transition           model/trunk/blocks.py:79-96              TransitionBlock.forward
 *  sf_linear               model/layers/primitives.py:328-372       Linear.forward (post_op, residual)
 *  sf_pair_logits          model/trunk/blocks.py:745-749            SingleActUpdate pair-logit projection
 */
#ifndef SPARSEFOLD_B200_H_
#define SPARSEFOLD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sf_stream_t; /* == cudaStream_t */

enum sf_dtype { SF_F32 = 0, SF_BF16 = 1 };

enum sf_status {
  SF_OK = 0,
  SF_ERR_ARG = 1,         /* bad shape, null pointer, unsupported combination */
  SF_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
  SF_ERR_WORKSPACE = 3,   /* workspace too small */
  SF_ERR_DEVICE = 4,      /* current device is not sm_100 */
  SF_ERR_TIMEOUT = 5      /* a bounded device-side wait gave up (kernel set an error flag) */
};

enum sf_post_op { SF_POST_NONE = 0, SF_POST_RELU = 1, SF_POST_SILU = 2, SF_POST_SIGMOID = 3 };

/* ---- runtime ------------------------------------------------------------ */
const char* sf_version(void);
/* Copies the calling thread's last error message into buf; returns its length. */
int sf_last_error(char* buf, size_t len);
/* SF_OK when the current device is an sm_100 part this build was compiled for. */
int sf_device_check(void);
/* Number of kernels this library launched since load (all threads). */
uint64_t sf_launch_count(void);
/* Reads (and with clear != 0 resets) the current device's status word: 0, or
 * SF_ERR_TIMEOUT when a kernel's bounded wait gave up.  Synchronises the device. */
int sf_device_status(uint32_t* out, int clear);
/* Self-test of the bounded device-side wait (no counterpart in the reference: it
 * exercises this library's failure detection).  Launches one warp that waits on an
 * mbarrier with a bound of `polls` polls (1 .. 2^22); with arrive == 0 nothing
 * ever arrives, the wait gives up, the kernel records SF_ERR_TIMEOUT in the status
 * word read by sf_device_status() and returns.  With arrive != 0 the barrier
 * completes and the status word is left unchanged. */
int sf_selftest_wait(uint32_t polls, int arrive, sf_stream_t stream);

/* ---- generic attention: sdpa.py:22-121 ---------------------------------
 * out[b,q,h,:] = softmax_k(scale * q.k + bias[b,h,q,k] + maskbias) @ v
 * where maskbias = -FLT_MAX when !mask_q[b,q] or !mask_k[b,k] or !mask_row[b].
 * Strides are in elements; the innermost (head-dim) axis is contiguous.
 * `bias` may broadcast over batch (bias_sb == 0).  If `gate` is non-null the
 * output is multiplied by sigmoid(gate) (same layout as out) — the gating of
 * GridSelfAttention._attention (blocks.py:288-289).                      */
typedef struct sf_attention_args {
  int dtype;
  int64_t batch, heads, q_len, k_len, head_dim;
  const void* q; int64_t q_sb, q_sh, q_sq;
  const void* k; int64_t k_sb, k_sh, k_sk;
  const void* v; int64_t v_sb, v_sh, v_sk;
  void* out; int64_t o_sb, o_sh, o_sq;
  const void* bias; int bias_dtype; int64_t b_sb, b_sh, b_sq;
  const uint8_t* mask_q; int64_t mq_sb;
  const uint8_t* mask_k; int64_t mk_sb;
  const uint8_t* mask_row;
  const void* gate; int64_t g_sb, g_sh, g_sq;
  float scale;
  int64_t value_dim;   /* head dim of v, out and gate; 0 = head_dim (sdpa.py allows Dv != Dqk) */
} sf_attention_args;
int sf_attention(const sf_attention_args* args, sf_stream_t stream);

/* ---- LayerNorm over the last axis (primitives.py:471-497), eps per call. */
int sf_layernorm(int dtype, const void* x, void* y, const float* weight, const float* bias,
                 int64_t rows, int64_t cols, float eps, sf_stream_t stream);

/* ---- Linear (primitives.py:328-372): y = post_op(x @ W + bias + residual).
 * x [rows][k], wt [n][k], y/residual [rows][n]; bias/residual may be null. */
int sf_linear(int dtype, const void* x, const void* wt, const float* bias, const void* residual,
              void* y, int64_t rows, int64_t k, int64_t n, int post_op, sf_stream_t stream);

/* ---- TriangleMultiplication (blocks.py:484-566) --------------------------
 * w_glu: [4][C][C] rows = (gate of a-channels, value of a-channels,
 *        gate of b-channels, value of b-channels); a-channel c is the
 *        reference projection channel 2c, b-channel c is 2c+1 (blocks.py:538).
 * w_out = output_projection^T, w_gate = gating_linear^T, both [C][C].        */
typedef struct sf_tri_mult_weights {
  const float* ln_w; const float* ln_b;          /* left_norm_input */
  const void* w_glu;                              /* [4C][C] */
  const float* center_w; const float* center_b;  /* center_norm */
  const void* w_out;                              /* [C][C] */
  const void* w_gate;                             /* [C][C] */
} sf_tri_mult_weights;

/* Row pitch of the channel-major buffers a_op, b_op and p: n rounded up to a
 * multiple of 8 elements (16-byte aligned rows).  Padding columns are zero. */
int64_t sf_pair_pitch(int64_t n);

/* Phase 1: x = LN(z); proj = sigmoid(x Wg) * (x Wv) * mask; writes the two
 * contraction operands so that phase 2 is always P[c,i,j] = sum_k A[c,i,k] B[c,j,k]:
 *   outgoing: A[c][i][k] = a[c,i,k], B[c][j][k] = b[c,j,k]   (rows = i, cols = k)
 *   incoming: A[c][i][k] = b[c,k,i], B[c][j][k] = a[c,k,j]   (stored transposed)
 * a_op / b_op are [C][n][sf_pair_pitch(n)] for the full device case. */
int sf_tri_mult_project(int dtype, const void* z, const uint8_t* mask, int64_t n, int incoming,
                        const sf_tri_mult_weights* w, void* a_op, void* b_op,
                        void* ws, size_t ws_bytes, sf_stream_t stream);
size_t sf_tri_mult_project_workspace(int dtype, int64_t n);
/* Phase 2: P[c][i][j] = sum_k A[c][i][k] * B[c][j][k]; A [C][rows][pitch(kdim)],
 * B [C][cols][pitch(kdim)], P [C][rows][pitch(cols)]. */
int sf_tri_mult_contract(int dtype, const void* a_op, const void* b_op, void* p,
                         int64_t channels, int64_t rows, int64_t cols, int64_t kdim, sf_stream_t stream);
/* Phase 3: z_out = z + (centerLN(P) W_out) * sigmoid(LN(z) W_gate); z_out may alias z. */
int sf_tri_mult_output(int dtype, const void* z, const void* p, int64_t rows, int64_t n,
                       const sf_tri_mult_weights* w, void* z_out,
                       void* ws, size_t ws_bytes, sf_stream_t stream);
size_t sf_tri_mult_output_workspace(int dtype, int64_t rows, int64_t n);

/* ---- GridSelfAttention (blocks.py:270-366), H heads of D = C / H --------
 * w_qkvg: [4][C][C] rows = q (h,d), k (h,d), v (h,d), gating_query;
 * w_bias: [H][C] pair_bias_projection^T; w_out: output_projection^T [C][C]. */
typedef struct sf_tri_attention_weights {
  const float* ln_w;        /* act_norm scale (no offset) */
  const void* w_qkvg;       /* [4C][C] */
  const void* w_bias;       /* [H][C] */
  const void* w_out;        /* [C][C] */
  int64_t heads;
} sf_tri_attention_weights;
/* Whole op on one device: z_out = z + GridSelfAttention(z); z_out may alias z. */
int sf_tri_attention(int dtype, const void* z, const uint8_t* mask, int64_t n, int transpose,
                     const sf_tri_attention_weights* w, void* z_out,
                     void* ws, size_t ws_bytes, sf_stream_t stream);
size_t sf_tri_attention_workspace(int dtype, int64_t n, int64_t heads);

/* ---- phases of the row-sharded pair track (bf16) --------------------------
 * The pair tensor is split by rows over P ranks (runtime/dist.py:173-235); each
 * rank owns `rows` pair rows starting at global row `row_offset`, all n columns.
 * The collectives between phases mirror the reference's choreography
 * (blocks.py:541-555, :320-346) and run in NCCL through the host.            */
/* Tri-mult projection of a row shard.  Outgoing: A, B are [rows][C][pitch(n)].
 * Incoming: A = b^T, B = a^T are [n][C][pitch(rows)] (send buffers of the
 * all-to-all / all-gather that assemble the K axis across ranks). */
int sf_tri_mult_project_rows(int dtype, const void* z, const uint8_t* mask, int64_t rows, int64_t n,
                             int64_t row_offset, int incoming, const sf_tri_mult_weights* w,
                             void* a_op, void* b_op, sf_stream_t stream);
/* P[i][c][j] = sum_k A[i][c][k] B[j][c][k] where each operand may hold K in
 * `chunks` equal pieces laid out [chunk][row][C][pitch(kdim/chunks)] (one per
 * source rank); chunk lengths must be multiples of 64 when chunks > 1. */
int sf_tri_mult_contract_chunked(int dtype, const void* a_op, int64_t chunks_a, const void* b_op,
                                 int64_t chunks_b, void* p, int64_t channels, int64_t rows, int64_t cols,
                                 int64_t kdim, sf_stream_t stream);
/* Query pitch qp of the attention buffers: K [nb][4][qp][32], Vt [nb][4][32][qp], Q (stored times
 * log2(e)/sqrt(32)) and G = sigmoid(gate) [nb][4][qp/32][4][32][8] (per group of 32 queries, four
 * [32 queries][8 channels] chunks), bias [qp][4][qp] (bias[q][h][k], rows gathered across ranks). */
int64_t sf_tri_attention_query_pitch(int64_t nq);
/* Pair bias of the local rows: bias[(r*4 + h)*ldb + s] = log2(e) * LN(z[r,s]) . W_b[h] in bf16
 * (blocks.py:317-320; stored in base-2 logit units, the form the attention core adds its scaled
 * Q K^T to). */
int sf_tri_attention_bias(int dtype, const void* z, int64_t rows, int64_t n, const sf_tri_attention_weights* w,
                          void* bias, int64_t ldb, sf_stream_t stream);
/* LN + q/k/v/gate projections of a z block [rows][cols]; transpose = attention
 * along columns (ending node).  With compute_bias the block's own positions
 * write the bias rows. */
int sf_tri_attention_project(int dtype, const void* z, int64_t rows, int64_t cols, int transpose,
                             int compute_bias, const sf_tri_attention_weights* w, void* q, void* k,
                             void* vt, void* g, void* bias, sf_stream_t stream);
/* Attention + gate + output projection + residual on the z block; batch_offset
 * is the global token index of the block's first attention row (row mask). */
int sf_tri_attention_core(int dtype, const void* q, const void* k, const void* vt, const void* g,
                          const void* bias, const uint8_t* mask, const void* z, void* z_out, int64_t rows,
                          int64_t cols, int transpose, int64_t batch_offset,
                          const sf_tri_attention_weights* w, sf_stream_t stream);

/* ---- TransitionBlock (blocks.py:79-96): y = x + swish(LN(x) W1a) * (LN(x) W1b) W2
 * w1: [2I][C] (first I rows = swish half), w2: [C][I]; y may alias x.        */
int sf_transition(int dtype, const void* x, const float* ln_w, const float* ln_b,
                  const void* w1, const void* w2, void* y, int64_t rows, int64_t c, int64_t inter,
                  void* ws, size_t ws_bytes, sf_stream_t stream);
size_t sf_transition_workspace(int dtype, int64_t rows, int64_t inter);

/* sf_transition for callers that cannot allocate device memory (no counterpart
 * in the reference).  Same arguments as sf_transition minus the workspace: the
 * scratch is a fixed array of sf_transition_noalloc_max_scratch() bytes
 * (16 MiB) inside the library, reserved on every GPU that loads it until exit.
 * Sizes whose sf_transition_workspace() exceeds it return SF_ERR_WORKSPACE.
 * The first call on a device looks up the array's device address (make it
 * before any stream capture).  All calls share the array, so calls that
 * overlap on the GPU race; the array needs no clearing between calls. */
int sf_transition_noalloc(int dtype, const void* x, const float* ln_w, const float* ln_b,
                          const void* w1, const void* w2, void* y, int64_t rows, int64_t c,
                          int64_t inter, sf_stream_t stream);
size_t sf_transition_noalloc_max_scratch(void);

/* ---- SingleActUpdate pair logits (blocks.py:745-749):
 * logits[h][i][j] = LN(z[i,j]) . W[h]; w: [H][C] (single_pair_logits_projection^T). */
int sf_pair_logits(int dtype, const void* z, const float* ln_w, const float* ln_b, const void* w,
                   void* logits, int64_t rows, int64_t n, int64_t c, int64_t heads,
                   void* ws, size_t ws_bytes, sf_stream_t stream);
size_t sf_pair_logits_workspace(int dtype, int64_t rows, int64_t n, int64_t c);

/* ---- diffusion-transformer and MSA helpers ----------------------------- */
/* y = scale * LN(x) + bias (norm without affine): AdaptiveLayerNorm with
 * single_cond (model/diffusion/transformer.py:80-93); x, y [rows][cols]; scale, bias
 * [cond_rows][cols], repeated every cond_rows rows of x (one conditioning for every
 * diffusion sample; rows must be a multiple of cond_rows). */
int sf_adaln(int dtype, const void* x, const void* scale, const void* bias, void* y, int64_t rows,
             int64_t cols, int64_t cond_rows, sf_stream_t stream);
/* out[e] = base[e] + u[e] * gate[e % gate_period] (base may be null): AdaptiveZeroInit gating
 * and residual (transformer.py:138-154, :345, :585), MSAAttention gate (trunk/blocks.py:182-183);
 * n must be a multiple of gate_period. */
int sf_gated_residual(int dtype, const void* base, const void* u, const void* gate, void* out, int64_t n,
                      int64_t gate_period, sf_stream_t stream);
/* out[b][i][:] = mask[i] ? src[b][idx[i]][:] : 0 — atom_layout.convert
 * (schema/atom_layout.py:52-83) for the atom key windows (transformer.py:671-673). */
int sf_gather_rows(int dtype, const void* src, int64_t batch, int64_t src_rows, const int32_t* idx,
                   const uint8_t* mask, int64_t n_out, int64_t cols, void* out, sf_stream_t stream);
/* x[r][:] = 0 where !mask[r] (masked_fill of the OPM projections, trunk/blocks.py:645-647). */
int sf_mask_rows(int dtype, void* x, const uint8_t* mask, int64_t rows, int64_t cols, sf_stream_t stream);
/* y = softmax(x + key_bias) over the last axis (MSAAttention weights, trunk/blocks.py:163-170). */
int sf_softmax_rows(int dtype, const void* x, const float* key_bias, void* y, int64_t rows, int64_t k,
                    int64_t ldy, sf_stream_t stream);
/* out[r][i] = swish(h[r][i]) * h[r][I + i]: the GLU of the diffusion transitions
 * (layers/primitives.py:624-631, diffusion/transformer.py:218-228). */
int sf_swiglu(int dtype, const void* h, void* out, int64_t rows, int64_t inter, sf_stream_t stream);
/* Batched strided transpose out[ob(b)+c*os_c+r] = in[ib(b)+r*is_r+c], b = (b1 < nb1, b2 < nb2),
 * ib = b1*ib1 + b2*ib2, ob = b1*ob1 + b2*ob2 (layout changes of the einsums at
 * trunk/blocks.py:179 and :667). */
int sf_transpose(int dtype, const void* in, void* out, int64_t nb1, int64_t nb2, int64_t rows, int64_t cols,
                 int64_t ib1, int64_t ib2, int64_t is_r, int64_t ob1, int64_t ob2, int64_t os_c,
                 sf_stream_t stream);
/* OuterProductMean normaliser norm[i][j] = 1/(1e-3 + sum_m mask[m,i] mask[m,j])
 * (trunk/blocks.py:683-688); mask [n_seq][n_res] uint8, norm [n_res][n_res] fp32. */
int sf_opm_norm(int dtype, const uint8_t* mask, int64_t n_seq, int64_t n_res, float* norm, void* ws,
                size_t ws_bytes, sf_stream_t stream);
size_t sf_opm_norm_workspace(int64_t n_seq, int64_t n_res);
/* out[(i*n+j)][a*d+b] = O[i*d+a][j*d+b]: the outer-product blocks as rows for the
 * output projection (trunk/blocks.py:667-669); O row pitch `pitch`. */
int sf_opm_repack(int dtype, const void* o, int64_t pitch, int64_t n_res, int64_t d, void* out,
                  sf_stream_t stream);
/* x[r][:] *= s[r] (the OPM normaliser, trunk/blocks.py:689). */
int sf_scale_rows(int dtype, void* x, const float* s, int64_t rows, int64_t cols, sf_stream_t stream);
/* dst[b*dbs + r*drs + c] = src[b*sbs + r*srs + c] for nblk blocks of rows x width_bytes (all in bytes,
 * multiples of 16): the packing of the pair tensor between row and column shards around the all-to-all
 * of the ending-node attention (runtime/dist.py:477-565 reshard, trunk/blocks.py:335-346). */
int sf_copy_blocks(void* dst, const void* src, int64_t nblk, int64_t rows, int64_t width_bytes,
                   int64_t src_blk_stride, int64_t src_row_stride, int64_t dst_blk_stride,
                   int64_t dst_row_stride, sf_stream_t stream);
/* out[i][j][:] = left[i][:] + right[j][:] (+ addend[i][j][:] when not NULL), rows x cols x channels:
 * the sequence pair embedding left_single(target_feat_shard)[:, None] + right_single(target_feat)[None, :]
 * of Evoformer._get_seq_pair_embedding (trunk/network.py:195-212).  fp32 sum, rounded once. */
int sf_pair_outer_sum(int dtype, const void* left, const void* right, const void* addend, void* out,
                      int64_t rows, int64_t cols, int64_t channels, sf_stream_t stream);
/* out[p][:] = sum_k x[p][k] w[k][:] (+ residual[p][:] when not NULL) for `positions` rows of x [positions][k]:
 * the pair-side linear layers whose inputs are one-hot or 0/1 features, the relative-position encoding
 * (Evoformer._get_position_feat, trunk/network.py:188-193, k = 139) and the bond contact map
 * (Evoformer._get_bonds_act, :214-256, k = 1).  w is fp32 [k][channels] (the reference Linear's
 * input_shape + output_shape layout); channels 32, 64, 128 or 256.  Only nonzero x[p][k] contribute
 * (a zero feature skips its term), in increasing k, fp32 sums rounded once to dtype. */
int sf_pair_sparse_linear(int dtype, const void* x, const float* w, const void* residual, void* out,
                          int64_t positions, int64_t k, int64_t channels, sf_stream_t stream);
/* ---- Peer exchanges over NVLink (the all-to-all / all-gather of the row-sharded path,
 * runtime/dist.py:477-565, between the ranks of one box, one process per GPU) ----
 * sf_ipc_export: the CUDA IPC handle (CUDA_IPC_HANDLE_SIZE = 64 bytes) of the device
 * allocation holding ptr, and ptr's offset in it.  sf_ipc_import: ptr = a peer's allocation
 * mapped into this process (cudaIpcOpenMemHandle, peer access enabled; one mapping per
 * handle and device, reused) + offset.  sf_ipc_close_all unmaps every imported allocation. */
int sf_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int sf_ipc_import(const void* handle, uint64_t offset, void** ptr);
int sf_ipc_close_all(void);
/* Block q of src (block_bytes each, src_stride_bytes apart, q = 0 .. n-1) is written to
 * dsts_dev[q] + dst_offset_bytes with 16-byte stores from the SMs; dsts_dev is a device array
 * of n pointers (local or peer-mapped).  Everything a multiple of 16 bytes. */
int sf_scatter_peers(const void* src, void* const* dsts_dev, int32_t n, int64_t block_bytes,
                     int64_t src_stride_bytes, int64_t dst_offset_bytes, sf_stream_t stream);
/* After everything earlier on the stream: *flag = value (a peer's flag word, system-scope
 * release).  sf_peer_wait: the stream waits until flags[q] >= value (wrapping compare) for every
 * q != self, q < n <= 32, polling at most `polls` times (about 0.25 us apart); on timeout the
 * kernel records SF_ERR_TIMEOUT in sf_device_status() and returns. */
int sf_peer_signal(uint32_t* flag, uint32_t value, sf_stream_t stream);
int sf_peer_wait(const uint32_t* flags, int32_t n, int32_t self, uint32_t value, uint32_t polls,
                 sf_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARSEFOLD_B200_H_ */
