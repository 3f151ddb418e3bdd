/*
 * foldforge_b200 C ABI: B200 (sm_100a) kernels of FoldForge's Pairformer pair stack.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (`void*`, a
 * cudaStream_t; NULL = the legacy default stream) and returns an ffb_status. Entry points
 * enqueue work on the stream and return without synchronising the host, allocate nothing
 * (scratch space is passed in by the caller), and keep no state between calls other than
 * per-device caches (SM count, the device error word's address), so they are safe to
 * call from several host threads and to capture in a CUDA graph.
 *
 * Layouts (bf16 = IEEE bfloat16, row-major, last axis contiguous):
 *   pair  z      [B, N, N, c_z]    channels last, c_z = 128
 *   single s     [B, N, c_s]
 *   key mask     [B, N]            uint8, 1 = real token, 0 = padding
 * Each op returns its input PLUS its update (the engine classes own their residual).
 *
 * Device-side waits are bounded: a launch that cannot make progress records a code in a
 * per-device error word and exits; ffb_device_error() reads (and clears) it.
 *
 * The reference interfaces these entry points replace are the engine modules FoldForge
 * calls through its backend guard (src/foldforge/modules/engine/policy.py:85-101); each
 * declaration names the reference equations it computes.
 */
#ifndef FOLDFORGE_B200_H
#define FOLDFORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FFB_OK = 0,
  FFB_ERR_ARG = 1,         /* a pointer, size or stride the entry point cannot take */
  FFB_ERR_UNSUPPORTED = 2, /* a shape / dtype outside the kernels' range (the backend's refusal) */
  FFB_ERR_CUDA = 3,        /* a CUDA runtime error while enqueueing */
  FFB_ERR_DEVICE = 4       /* a device-side error word was set (see ffb_device_error) */
} ffb_status;

typedef enum { FFB_BF16 = 0, FFB_F32 = 1 } ffb_dtype;

/* Masked-position policy of the pair/single updates.
 * FFB_MASKED_COMPUTE: every position gets the reference equations' update, including
 *   padded ones (what FoldForge's legacy block computes, legacy/pairformer.py:191-229).
 * FFB_MASKED_ZERO: the update at every pair (i, j) with mask_i * mask_j == 0, and at
 *   every padded single row, is exactly 0 (the output equals the input there). */
typedef enum { FFB_MASKED_COMPUTE = 0, FFB_MASKED_ZERO = 1 } ffb_masked;

/* Library version (major * 10000 + minor * 100 + patch). */
int ffb_version(void);

/* Human-readable text of the last non-OK status returned on this host thread. */
const char* ffb_last_error(void);

/* Synchronises `stream`, then reads and clears the current device's error word. */
int ffb_device_error(int* code, void* stream);

/* LayerNorm over the last axis: y = (x - mean) / sqrt(var + eps) * gamma + beta.
 * x, y [rows, c] of `dtype`; gamma, beta fp32 [c] or NULL (affine skipped).
 * Replaces the engine `LayerNorm` op (src/foldforge/modules/engine/modules.py:230-238). */
int ffb_layernorm_fwd(const void* x, void* y, const float* gamma, const float* beta, int64_t rows, int c, float eps,
                      int dtype, void* stream);

/* Batched bf16 GEMM, D[b] = A[b] @ B[b]^T with fp32 accumulation on the tensor cores.
 * A [batch, m, k] (row stride lda, batch stride sa), B [batch, n, k] (ldb, sb), D [batch, m, n]
 * (ldd, sd) of d_dtype. Strides in elements; lda, ldb multiples of 8; k % 8 == 0.
 * epilogue: 0 store (+bias[n] fp32 if non-NULL); 1 residual: D = R + (acc + bias) * row_mask[m]
 * (R like D; row_mask uint8 [batch, m] or NULL); 2 SwiGLU over a/b rows interleaved in blocks
 * of 16 (D has n / 2 columns).
 * The plain projections of the single track (legacy/transformer.py:88-133). */
int ffb_gemm_bf16_nt(const void* a, const void* b, void* d, int batch, int m, int n, int k, int64_t lda,
                     int64_t ldb, int64_t ldd, int64_t sa, int64_t sb, int64_t sd, int d_dtype, const float* bias,
                     int epilogue, const void* residual, const uint8_t* row_mask, void* stream);

/* ---- Triangle multiplicative update (c_z = hidden = 128, bf16 activations).
 * Replaces the engine `TriangleMultiplication` (outgoing / incoming) as FoldForge calls it
 * (src/foldforge/modules/engine/modules.py:144-163); equations of
 * legacy/reference/triangle.py:19-50 with the engine weight names of
 * legacy/released.py:135-173.
 *
 * ffb_trimul_prepare packs the fp32 master weights (all [out, in] row-major, LayerNorm
 * vectors [128]) into `packed` (ffb_trimul_packed_bytes() bytes, 16-byte aligned). Run it
 * once per weight update; the forward pass only reads the packed image.
 * ffb_trimul_fwd: z, out [B, N, N, 128] bf16 (out may not alias z), mask [B, N] uint8,
 * workspace of ffb_trimul_workspace_bytes(B, N) bytes (256-byte aligned). */
size_t ffb_trimul_packed_bytes(void);
size_t ffb_trimul_workspace_bytes(int B, int N);
int ffb_trimul_prepare(const float* ln_w, const float* ln_b, const float* ln_out_w, const float* ln_out_b,
                       const float* to_left, const float* to_right, const float* to_left_gate,
                       const float* to_right_gate, const float* to_out, const float* to_gate, void* packed,
                       void* stream);
int ffb_trimul_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                   size_t workspace_bytes, int B, int N, int outgoing, int masked, void* stream);
/* The same with a subset of its three launches: `stages` bit 0 = projection (z -> L, R in
 * the workspace), bit 1 = contraction (L, R -> U), bit 2 = output (U, z -> out); 7 = all.
 * For profiling one launch, and for callers that move the workspace between stages. */
int ffb_trimul_fwd_stages(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                          size_t workspace_bytes, int B, int N, int outgoing, int masked, int stages, void* stream);

/* ---- Triangle attention, starting / ending node (c_z = 128, 4 heads x 32, AF3: no
 * projection biases, untransposed pair bias). Replaces the engine `TriangleAttention`
 * (model "af3") as FoldForge calls it (src/foldforge/modules/engine/modules.py:166-181);
 * equations of legacy/attention.py:108-171 and legacy/reference/attention.py:14-100.
 * ffb_triattn_prepare: fp32 master weights (ln_w, ln_b [128]; to_bias [4, 128]; to_query,
 * to_key, to_value, to_gate, to_out [128, 128]) -> `packed` (ffb_triattn_packed_bytes()).
 * ffb_triattn_fwd: as ffb_trimul_fwd, with workspace ffb_triattn_workspace_bytes(B, N). */
size_t ffb_triattn_packed_bytes(void);
size_t ffb_triattn_workspace_bytes(int B, int N);
int ffb_triattn_prepare(const float* ln_w, const float* ln_b, const float* to_bias, const float* to_query,
                        const float* to_key, const float* to_value, const float* to_gate, const float* to_out,
                        void* packed, void* stream);
int ffb_triattn_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                    size_t workspace_bytes, int B, int N, int starting, int masked, void* stream);
/* `stages` bit 0 = projection (z -> Q, K, V^T, bias), bit 1 = attention (-> o), bit 2 =
 * gated output projection (o, z -> out); 7 = all. */
int ffb_triattn_fwd_stages(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                           size_t workspace_bytes, int B, int N, int starting, int masked, int stages, void* stream);

/* ---- Pair transition (c_z = 128, factor 4), fused LayerNorm -> expand -> SwiGLU ->
 * squeeze -> residual. Replaces the engine `Transition(128, 4)` as FoldForge calls it
 * (src/foldforge/modules/engine/modules.py:133-141); equations of legacy/primitives.py:20-37
 * and legacy/reference/transition.py:28-59 (expand_a / expand_b = legacy/released.py:211-224).
 * ffb_transition_prepare: ln_w, ln_b [128], expand_a, expand_b [512, 128], squeeze [128, 512]
 * fp32 -> `packed` (ffb_transition_packed_bytes()). ffb_transition_fwd needs no workspace.
 * `mask` may be NULL when masked == FFB_MASKED_COMPUTE. */
size_t ffb_transition_packed_bytes(void);
int ffb_transition_prepare(const float* ln_w, const float* ln_b, const float* expand_a, const float* expand_b,
                           const float* squeeze, void* packed, void* stream);
int ffb_transition_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int N, int masked,
                       void* stream);

/* ---- Single-track attention with pair bias (c_s = 384, 16 heads x 24, c_z = 128).
 * Replaces the engine `AttentionPairBias` of the Pairformer block; equations of
 * legacy/pairformer.py:204-226 and legacy/transformer.py:88-133 with the engine weight
 * names of legacy/released.py:281-315 (the pair LayerNorm has no offset).
 * ffb_apb_prepare: ln_single_w/_b [384], to_query [384, 384], query_bias [384], to_key,
 * to_value, to_gate, to_out [384, 384], ln_pair_w [128], to_bias [16, 128] (fp32).
 * ffb_apb_fwd: s, out [B, N, 384] bf16; z [B, N, N, 128] bf16 (the pair AFTER the pair
 * track); extra_pair_bias [B, 16, N, N] (extra_dtype FFB_BF16 / FFB_F32) or NULL;
 * gate_bias is added to the gate logits (0 for AF3). */
size_t ffb_apb_packed_bytes(void);
size_t ffb_apb_workspace_bytes(int B, int N);
int ffb_apb_prepare(const float* ln_single_w, const float* ln_single_b, const float* to_query,
                    const float* query_bias, const float* to_key, const float* to_value, const float* to_gate,
                    const float* to_out, const float* ln_pair_w, const float* to_bias, void* packed, void* stream);
int ffb_apb_fwd(const void* s, const void* z, const uint8_t* mask, const void* packed, const void* extra_pair_bias,
                int extra_dtype, float gate_bias, void* out, void* workspace, size_t workspace_bytes, int B, int N,
                int masked, void* stream);

/* ---- Single transition (c_s = 384, factor 4). Same equations as the pair transition.
 * ffb_single_transition_prepare: ln_w, ln_b [384], expand_a, expand_b [1536, 384],
 * squeeze [384, 1536] fp32. ffb_single_transition_fwd: s, out [B, N, 384] bf16. */
size_t ffb_single_transition_packed_bytes(void);
size_t ffb_single_transition_workspace_bytes(int B, int N);
int ffb_single_transition_prepare(const float* ln_w, const float* ln_b, const float* expand_a,
                                  const float* expand_b, const float* squeeze, void* packed, void* stream);
int ffb_single_transition_fwd(const void* s, const uint8_t* mask, const void* packed, void* out, void* workspace,
                              size_t workspace_bytes, int B, int N, int masked, void* stream);

/* The single transition for callers that cannot allocate device memory when they run it
 * (a host whose device memory belongs to its own pool or arena, a pipeline that allocates
 * only at start-up). No counterpart in the reference: it exists for those callers only.
 * Same arguments and result as ffb_single_transition_fwd minus the workspace, which is a
 * fixed 3,932,160-byte array inside the library that every GPU loading the library keeps
 * until the process exits. B * N must be at most 1024 tokens (larger calls return
 * FFB_ERR_UNSUPPORTED). The array's device address is looked up on a device's first call,
 * with that device current: make the first call before any stream capture. All calls share
 * the array, so calls whose GPU work overlaps race and must be serialised by the caller.
 * Allocates nothing. */
int ffb_single_transition_fwd_noalloc(const void* s, const uint8_t* mask, const void* packed, void* out, int B, int N,
                                      int masked, void* stream);

/* ---- Row-sharded pieces (axial parallelism over the GPUs of one box; B = 1). A rank holds
 * pair rows [row0, row0 + R) of the N x N pair z [R, N, 128] (bf16), or of its transpose
 * for the column-wise ops (TriMul incoming = outgoing on z^T with the left / right weights
 * swapped; TriAttn ending = starting on z^T with the untransposed bias). The host moves data
 * between the pieces with NCCL (all-gather over rows, all-to-all transposes); no new
 * reference interface corresponds to these: FoldForge has no multi-GPU Pairformer.
 * Layouts: TriMul L, R, and the gathered right operand [rows][128][Np] bf16 (Np = N rounded
 * up to 8), U [128][R][Np] bf16, statistics [R][N] float2 (ffb_trimul_shard_out's `ustats` is unused and
 * may be null: the output kernel takes u's statistics itself); TriAttn Q, K [R][4][N][32],
 * V^T [R][4][32][Np], bias rows [R][4][Np] (gathered: [N][4][Np], rows = queries), o [R][N][128];
 * single-track pair-bias rows [R][16][N] fp32 (gathered: [N][16][N]). Weights are the
 * ffb_*_prepare images. Status codes as elsewhere. */
int ffb_trimul_shard_proj(const void* z, const uint8_t* mask, const void* packed, void* left, void* right,
                          void* zstats, int R, int N, int row0, void* stream);
int ffb_trimul_shard_contract(const void* left, const void* right_all, void* u, int R, int N, void* stream);
int ffb_trimul_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* u, const void* zstats,
                         void* ustats, void* out, int R, int N, int row0, int masked, void* stream);
int ffb_triattn_shard_proj(const void* z, const void* packed, void* q, void* k, void* vt, void* bias_rows, int R, int N,
                           void* stream);
int ffb_triattn_shard_attn(const void* q, const void* k, const void* vt, const void* bias_all, const uint8_t* mask,
                           void* o, int R, int N, int row0, void* stream);
int ffb_triattn_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* o, void* out, int R, int N,
                          int row0, int masked, void* stream);
int ffb_transition_shard_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, int R, int N, int row0,
                             int masked, void* stream);
int ffb_apb_shard_pair_bias(const void* z, const void* packed, void* pb_rows, int R, int N, void* stream);
size_t ffb_apb_single_workspace_bytes(int N);
int ffb_apb_shard_single(const void* s, const uint8_t* mask, const void* packed, const void* pb_all,
                         const void* extra_pair_bias, int extra_dtype, float gate_bias, void* out, void* workspace,
                         size_t workspace_bytes, int N, int masked, void* stream);
/* The rank's rows [row0, row0 + R) of the single track's attention with pair bias, computed
 * from its OWN pair-bias rows pb_rows [R][16][N] (fp32, ffb_apb_shard_pair_bias): the
 * projection runs over all N tokens of the replicated s, the attention for the R queries;
 * out_rows [R][384] bf16 = s rows + the update (the rank's rows, to be all-gathered). Replaces
 * the all-gather of the [N][16][N] pair bias that ffb_apb_shard_single needs. Workspace:
 * ffb_apb_single_workspace_bytes(N). */
int ffb_apb_shard_single_rows(const void* s, const uint8_t* mask, const void* packed, const void* pb_rows,
                              float gate_bias, void* out_rows, void* workspace, size_t workspace_bytes, int N,
                              int row0, int R, int masked, void* stream);

/* ---- Row-shard exchanges over NVLink peer memory (one rank per GPU of one box). Buffers
 * are plain device allocations shared through CUDA IPC handles (no multicast object):
 * ffb_p2p_alloc allocates and zeroes `bytes` on the current device and writes the IPC handle
 * (ffb_p2p_handle_bytes() bytes) to `handle`; a peer maps it with ffb_p2p_open and unmaps it
 * with ffb_p2p_close; the owner frees it with ffb_p2p_free once every peer has closed it.
 * ffb_shard_transpose_p2p: x = this rank's pair rows [R][N][128] bf16 (N = P R, row0 = rank R);
 * pair (i, q R + a) is written to rank q's buffer dst_ptrs[q] at [a][row0 + i] (the rows of
 * z^T rank q holds). ffb_shard_gather_p2p: `bytes` (a multiple of 16) from src are written to
 * every rank's buffer dst_ptrs[q] at offset rank * bytes. Both end by publishing a new epoch
 * (counted in this rank's `sync` words, two uint32 zeroed at allocation) into slot [rank] of
 * every rank's flag array (flag_ptrs[q]: P uint32); ffb_shard_wait_p2p makes the stream wait
 * until every slot of this rank's `flags` has reached this rank's epoch, for at most
 * `limit_us` microseconds of GPU wall-clock time (<= 0: 2 s): a peer that never signals sets
 * the device error word (code 106) and the stream goes on instead of hanging.
 * dst_ptrs and flag_ptrs are device arrays of P uint64 addresses (peers' mapped addresses,
 * this rank's own). Every rank issues the same sequence of exchanges; consecutive exchanges
 * must write different buffers. P <= 8. */
int ffb_p2p_handle_bytes(void);
int ffb_p2p_alloc(size_t bytes, void** ptr, void* handle);
int ffb_p2p_open(const void* handle, void** ptr);
int ffb_p2p_close(void* ptr);
int ffb_p2p_free(void* ptr);
int ffb_shard_transpose_p2p(const void* x, const void* dst_ptrs, const void* flag_ptrs, void* sync, int R, int N,
                            int row0, int rank, int P, void* stream);
int ffb_shard_gather_p2p(const void* src, size_t bytes, const void* dst_ptrs, const void* flag_ptrs, void* sync,
                         int rank, int P, void* stream);
int ffb_shard_wait_p2p(const void* flags, const void* sync, int P, int64_t limit_us, void* stream);

/* Channel-sharded TriMul contraction (P >= 4 ranks move less data this way than by gathering
 * the right operand): rank q owns channels [q C, (q + 1) C), C = 128 / P.
 * ffb_shard_rows_p2p mode 0: L or R rows [R][128][Np] of this rank -> every rank's
 * [C][N][Np] buffer (its channels, all rows); mode 1: U [C][N][Np] of this rank's channels ->
 * every rank's [128][R][Np] buffer (its rows, all channels). Signalling as above.
 * ffb_trimul_channel_contract: U[c] = L[c] R[c]^T for C channels, L, R, U [C][N][Np] bf16. */
int ffb_shard_rows_p2p(const void* src, int mode, int R, int N, const void* dst_ptrs, const void* flag_ptrs, void* sync,
                       int rank, int P, void* stream);
int ffb_trimul_channel_contract(const void* left, const void* right, void* u, int C, int N, void* stream);

/* ---- fp32 precision, and widths the tcgen05 kernels are not built for (FP32 SIMT cores).
 * The same ops with fp32 activations end to end (FoldForge's "fp32" precision,
 * modules/engine/configure.py:35-70) and any widths (e.g. the template stack's c_z = 64): fp32
 * LayerNorms, FFMA GEMMs with fp32 accumulation, softmax with expf. Weights are the engine's
 * fp32 matrices in their natural [out, in] layout, passed as a HOST array of device pointers
 * in the order listed; nothing is packed. Workspaces of the *_f32_workspace_bytes size,
 * 256-byte aligned; out may not alias the input; mask [B, N] uint8 is required. Each replaces
 * the same engine op as its bf16 counterpart above (TriangleMultiplication, TriangleAttention,
 * Transition, AttentionPairBias; src/foldforge/modules/engine/modules.py:133-181).
 * trimul weights: ln_w, ln_b [c], ln_out_w, ln_out_b [h], to_left, to_right, to_left_gate,
 *   to_right_gate [h, c], to_out [c, h], to_gate [c, c].
 * triattn weights: ln_w, ln_b [c], to_bias [H, c], to_query, to_key, to_value, to_gate [H d, c],
 *   to_out [c, H d]; d <= 64.
 * transition weights: ln_w, ln_b [c], expand_a, expand_b [n c, c], squeeze [c, n c]; `pair` 1:
 *   x [B, N, N, c] with the pair mask, 0: x [B, N, c] with the token mask.
 * apb weights: ln_single_w, ln_single_b [c_s], to_query [c_s, c_s], to_query_b [c_s], to_key,
 *   to_value, to_gate, to_out [c_s, c_s], ln_pair_w [c_z], to_bias [H, c_z]; extra_bias
 *   [B, H, N, N] fp32 or NULL; c_s / H <= 64. */
size_t ffb_trimul_f32_workspace_bytes(int B, int N, int c, int h);
int ffb_trimul_fwd_f32(const float* z, const uint8_t* mask, const float* const* weights, float* out, void* workspace,
                       size_t workspace_bytes, int B, int N, int c, int h, int outgoing, int masked, void* stream);
size_t ffb_triattn_f32_workspace_bytes(int B, int N, int c, int H, int d);
int ffb_triattn_fwd_f32(const float* z, const uint8_t* mask, const float* const* weights, float* out, void* workspace,
                        size_t workspace_bytes, int B, int N, int c, int H, int d, int starting, int masked,
                        void* stream);
size_t ffb_transition_f32_workspace_bytes(int64_t rows, int c, int n);
int ffb_transition_fwd_f32(const float* x, const uint8_t* mask, const float* const* weights, float* out,
                           void* workspace, size_t workspace_bytes, int B, int N, int c, int n, int pair, int masked,
                           void* stream);
size_t ffb_apb_f32_workspace_bytes(int B, int N, int cs, int cz, int H);
int ffb_apb_fwd_f32(const float* s, const float* z, const uint8_t* mask, const float* const* weights,
                    const float* extra_bias, float gate_bias, float* out, void* workspace, size_t workspace_bytes,
                    int B, int N, int cs, int cz, int H, int masked, void* stream);

/* ---- MSA module: AF3's MSA-stack block pieces (c_m = 64, c_z = 128; bf16 activations, fp32
 * accumulation on the tensor cores). Each replaces the engine class FoldForge's
 * graph.EvoformerBlock builds (src/foldforge/modules/engine/graph.py:237-309):
 * ffb_opm_* the engine OuterProductMean (modules/engine/modules.py:184-210; AF3 form:
 * legacy/reference/attention.py:57-74), ffb_pwa_* the engine MSAPairWeightedAveraging
 * (modules.py:213-227; legacy/attention.py:174-229), ffb_transition_gemm_* the engine
 * Transition at widths the fused pair kernel does not take (the MSA transition).
 * ffb_opm_prepare: fp32 ln_w, ln_b [64], to_left, to_right [32, 64], to_out_w [128, 1024]
 * (column c 32 + e), to_out_b [128] -> packed (ffb_opm_packed_bytes()).
 * ffb_opm_fwd: msa [B, S, N, 64] bf16, row_mask [B, S, N] uint8 -> delta [B, N, N, 128] bf16, the
 * RAW update (sum_{c,e} sum_s L[s,i,c] R[s,j,e] W[f, c 32 + e] + b[f]) / d(n_ij), n_ij = sum_s
 * m_si m_sj, d(n) = n + count_offset (AF3: 1e-3), or max(n, 1) when count_offset < 0. Workspace
 * ffb_opm_workspace_bytes(S, N) (per batch; batches run in turn).
 * ffb_pwa_prepare: fp32 ln_msa_w, ln_msa_b [64], ln_pair_w [128], to_bias [8, 128], to_value,
 * to_gate, to_out [64, 64] -> packed (ffb_pwa_packed_bytes()).
 * ffb_pwa_fwd: out = msa + W_o (sigmoid(W_g LN(m)) * o), o[s,i,h] = sum_j softmax_j(W_b LN(z)[i,j]
 * - 1e9 (1 - key_mask[j])) (W_v LN(m))[s,j,h]; msa, out [B, S, N, 64], pair [B, N, N, 128] bf16,
 * key_mask [B, N] uint8 (a column is a key when some MSA row has it); out may not alias msa.
 * ffb_transition_gemm_*: x + W_sq(silu(W_a LN(x)) * W_b LN(x)) over `rows` rows of c channels
 * (c a multiple of 8, n c of 16), unmasked; fp32 weights ln_w, ln_b [c], expand_a, expand_b
 * [n c, c], squeeze [c, n c]; packed 256-byte aligned. */
size_t ffb_opm_packed_bytes(void);
size_t ffb_opm_workspace_bytes(int S, int N);
int ffb_opm_prepare(const float* ln_w, const float* ln_b, const float* to_left, const float* to_right,
                    const float* to_out_w, const float* to_out_b, void* packed, void* stream);
int ffb_opm_fwd(const void* msa, const uint8_t* row_mask, const void* packed, void* delta, void* workspace,
                size_t workspace_bytes, int B, int S, int N, float count_offset, void* stream);
size_t ffb_pwa_packed_bytes(void);
size_t ffb_pwa_workspace_bytes(int S, int N);
int ffb_pwa_prepare(const float* ln_msa_w, const float* ln_msa_b, const float* ln_pair_w, const float* to_bias,
                    const float* to_value, const float* to_gate, const float* to_out, void* packed, void* stream);
int ffb_pwa_fwd(const void* msa, const void* pair, const uint8_t* key_mask, const void* packed, void* out,
                void* workspace, size_t workspace_bytes, int B, int S, int N, void* stream);
size_t ffb_transition_gemm_packed_bytes(int c, int n);
size_t ffb_transition_gemm_workspace_bytes(int64_t rows, int c, int n);
int ffb_transition_gemm_prepare(const float* ln_w, const float* ln_b, const float* expand_a, const float* expand_b,
                                const float* squeeze, int c, int n, void* packed, void* stream);
int ffb_transition_gemm_fwd(const void* x, const void* packed, void* out, void* workspace, size_t workspace_bytes,
                            int64_t rows, int c, int n, void* stream);

/* ---- Token diffusion transformer block (AF3 TokenDiT: c = 768, 16 heads x 48, conditioning
 * 384, pair 128, SwiGLU factor 2; replaces the engine TokenDiT block of
 * src/foldforge/modules/engine/transformers.py:31-125, algorithm legacy/transformer.py:28-294).
 * bf16 activations. Per block: ffb_dit_prepare packs the 23 fp32 weights, given as a HOST
 * array of device pointers in the engine schema's order: attention.ada_ln_in.{ln_cond.weight,
 * to_scale.weight, to_scale.bias, to_bias.weight}, attention.{to_query.weight, to_query.bias,
 * to_key.weight, to_value.weight, to_gate.weight, to_scale.weight, to_scale.bias,
 * to_out.weight, ln_pair.weight, to_bias.weight}, transition.ada_ln_in.{ln_cond.weight,
 * to_scale.weight, to_scale.bias, to_bias.weight}, transition.{expand_a.weight,
 * expand_b.weight, squeeze.weight, to_scale.weight, to_scale.bias}. Per fold (a fixed
 * conditioning): ffb_dit_condition fills the block's tables (ffb_dit_tables_bytes(L)) from
 * cond [L][384] and pair [L][L][128] (bf16): AdaLN scale / shift, output gates, pair logits.
 * Per sampler step: ffb_dit_fwd maps x [S][L][768] to out = the block's output (out must not
 * alias x); mask [L] (uint8, 0 = padding: keys masked with the replaced logit -1e9). */
size_t ffb_dit_packed_bytes(void);
int ffb_dit_prepare(const float* const* weights, void* packed, void* stream);
size_t ffb_dit_tables_bytes(int L);
size_t ffb_dit_condition_workspace_bytes(int L);
int ffb_dit_condition(const void* cond, const void* pair, const void* packed, void* tables, void* workspace,
                      size_t workspace_bytes, int L, void* stream);
size_t ffb_dit_workspace_bytes(int S, int L);
int ffb_dit_fwd(const void* x, const uint8_t* mask, const void* packed, const void* tables, void* out, void* workspace,
                size_t workspace_bytes, int S, int L, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FOLDFORGE_B200_H */
