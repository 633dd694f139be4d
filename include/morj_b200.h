/*
 * morj_b200: C-ABI of the B200 (sm_100a) tree-prefill kernels behind the lean engine's forward over a token tree.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed as void*), launches
 * asynchronously on that stream, allocates no device memory and returns a status code (0 on success). It never
 * throws or aborts across the ABI. `morj_last_error()` describes the most recent failure of the calling thread.
 * BF16 tensors are row-major with the leading dimension given in elements.
 *
 * Reference interfaces replaced (ALERIA-ML/MORJ, aleria_judge/lean_core.py):
 *   morj_gemm_bf16            torch.matmul (cuBLAS) at lean_core.py:670,682,685,686,701,708,729,733
 *   morj_gemm_bf16 (GEGLU)    the gate-up matmul + flashinfer.activation.gelu_tanh_and_mul, lean_core.py:685,733
 *   morj_gemm_qkv_rope        the QKV matmul + Triton _qkv_post, lean_core.py:670-674, 701-704, 708-712
 *   morj_rope_table           the per-step RoPE cos / sin tables, lean_core.py:636-640 (kept per model, by position)
 *   morj_embed_rmsnorm        embedding gather * embed_scale + image feature rows + flashinfer.rmsnorm,
 *                             lean_core.py:641-653
 *   morj_qkv_post             Triton _qkv_post, lean_core.py:234-277 (launches 672-674, 702-704, 710-712) with the
 *                             RoPE tables of lean_core.py:636-640
 *   morj_tree_attention       FlashInfer BatchPrefillWithPagedKVCacheWrapper plan()/run(), lean_core.py:609-635,
 *                             677-681, 723-728
 *   morj_attn_epilogue        Triton _attn_epilogue, lean_core.py:290-302 (launches 684, 732)
 *   morj_mlp_epilogue         Triton _mlp_epilogue, lean_core.py:305-320 (launches 689, 734)
 *   morj_label_head           final flashinfer.rmsnorm + label-row logits + softcap + per-branch softmax,
 *                             lean_core.py:558-561 with the norm of 692/736
 *   morj_gather_rows          x[rows] / hn[rows] gathers, lean_core.py:692,708,730
 *   morj_scatter_rows         K/V head copy into pool slots (_fill_head), lean_core.py:594-597
 *   morj_tree_build / morj_tree_layout / morj_plan_pass
 *                             the host planner: Tree.__init__ and Tree.plan_pass (with _depth_first, the step cut and
 *                             the liveness slot allocator), lean_core.py:38-83, 120-231
 */
#ifndef MORJ_B200_H
#define MORJ_B200_H

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MORJ_OK 0
#define MORJ_ERR_ARG 1      /* invalid argument (shape, alignment, null pointer) */
#define MORJ_ERR_CUDA 2     /* a CUDA runtime/driver call failed */
#define MORJ_ERR_OOM 3      /* out of device memory (never raised by calls that allocate nothing) */
#define MORJ_ERR_TIMEOUT 4  /* a kernel's bounded wait ran out (see morj_device_error) */
#define MORJ_ERR_UNSUPPORTED 5
#define MORJ_ERR_INTERNAL 6 /* an internal consistency check failed (the reference raises AssertionError there) */

/* GEMM epilogues */
#define MORJ_EPI_STORE 0 /* C[M,N] = bf16(A[M,K] . B[N,K]^T) */
#define MORJ_EPI_GEGLU 1 /* B rows interleaved in 128-row blocks (gate block, up block, ...); C[M,N/2] =
                            bf16(gelu_tanh(bf16(gate)) * bf16(up)) */
#define MORJ_EPI_QKV_D128 2 /* internal: the fused QKV epilogue of morj_gemm_qkv_rope, 128-wide heads */
/* Kernel choice, or-ed into morj_gemm_bf16's epilogue argument or morj_gemm_qkv_rope's has_v argument (default:
 * chosen per shape): the one-CTA kernel (128-row tiles) or the SM-pair kernel (256-row tiles,
 * tcgen05.mma.cta_group::2 over a 2-CTA cluster). */
#define MORJ_GEMM_FORCE_PAIR 0x100
#define MORJ_GEMM_FORCE_SINGLE 0x200
#define MORJ_EPI_QKV_D64 3  /* internal: the same, 64-wide heads */

/* Library version (major * 10000 + minor * 100 + patch). */
int morj_version(void);

/* Message of the calling thread's most recent failing call ("" if none). */
const char* morj_last_error(void);

/* Read (and clear, when `clear` != 0) the device error word that kernels set when a bounded wait runs out or a
 * precondition fails on the device; synchronises `stream`. *code = 0 means no kernel reported a failure. */
int morj_device_error(int* code, int clear, void* stream);

/* C = A . B^T with FP32 accumulation (tcgen05, TMEM accumulators, TMA-fed shared-memory ring).
 * A: [M, K] (lda), B: [N, K] (ldb), C: [M, N] (ldc) or [M, N/2] for MORJ_EPI_GEGLU.
 * Requires K % 8 == 0, lda/ldb/ldc % 8 == 0, 16-byte aligned pointers, N % 16 == 0 (N % 256 == 0 for GEGLU). */
int morj_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M, int N,
                   int K, int epilogue, void* stream);

/* Split-tile workspace of the SM-pair GEMM kernel (an addition; the reference's cuBLAS calls have no counterpart).
 * With a workspace registered for a stream, the pair-kernel GEMMs launched on that stream (morj_gemm_bf16,
 * morj_gemm_qkv_rope, morj_gemm_bf16_peer and morj_gemm_norm_epilogue_noalloc) share the k-blocks of the tiles that
 * do not fill a whole wave of SM pairs evenly between all pairs: a tile cut between two pairs sends the FP32 partial
 * of its first k-blocks through the workspace. Without one, every tile is computed whole (same results up to FP32
 * summation order). The memory is the caller's: at least morj_gemm_workspace_bytes() bytes (about 19 MB on a
 * 148-SM B200), 256-byte aligned, used by one stream only (launches on one stream run in order; two streams must
 * not share a workspace). morj_gemm_workspace_set zeroes the workspace's flags on `stream` and replaces any earlier
 * registration for (current device, stream); ptr = NULL removes it. morj_gemm_workspace_remove drops every
 * registration of `ptr` (call it before freeing the memory). At most 64 registrations. The same workspace lets
 * morj_gemm_bf16 run M <= 16 rows (plain and GeGLU epilogues; MORJ_GEMM_FORCE_* unset) on a weight-streaming kernel
 * that cuts every tile's K range over all SMs and adds the pieces' FP32 partials in k order through the workspace
 * (see morj_gemm_skinny_walk); without a workspace such calls take the tiled kernels. */
int morj_gemm_workspace_bytes(unsigned long long* bytes);
int morj_gemm_workspace_set(void* stream, void* ptr, unsigned long long bytes);
int morj_gemm_workspace_remove(const void* ptr);

/* The split schedule (host function, no device access): the work items pair `pair` of `pairs` walks for a GEMM of
 * `tiles` tiles of `kblocks` k-blocks, in order, as (tile, first k-block, end k-block, kind) int quadruples, kind
 * 0 = whole tile, 1 = first k-blocks of a cut tile (partial to the workspace), 2 = last k-blocks (adds the partial,
 * then the epilogue). Returns the number of items, -1 on bad arguments or when cap is too small. */
int morj_gemm_split_walk(int tiles, int pairs, int kblocks, int pair, int* items, int cap);

/* The schedule of the weight-streaming kernel morj_gemm_bf16 runs for M <= 16 rows (host function, no device
 * access): the (tile, k-block) units of `tiles` tiles of `kblocks` k-blocks, tile-major, cut into `ctas` contiguous
 * ranges; CTA `cta` walks, in order, (tile, first k-block, end k-block, piece, pieces) int quintuples: its piece of
 * each tile it touches and the tile's piece count. Returns the number of items, -1 on bad arguments (ctas must not
 * exceed tiles x kblocks) or when cap is too small. */
int morj_gemm_skinny_walk(int tiles, int kblocks, int ctas, int cta, int* items, int cap);

/* The QKV projection with the head epilogue fused: [q | k | v] = A . W^T (W: [N, K] rows q heads, k heads, v heads if
 * has_v; N = (hq + (1 + has_v) * hk) * d), each head RMSNorm'ed over the BF16-rounded projection (q, k weighted;
 * v unweighted), rounded, RoPE'd (q, k) and written straight to q_out[row, hq, d] and pool row slots[row] of
 * k_pool / v_pool. has_v = 0 (full-attention layers): V = the unweighted norm of the K projection. hq = 0 or hk = 0
 * give the K/V-only and q-only calls. Equivalent to morj_gemm_bf16 followed by morj_qkv_post, without the
 * intermediate [M, N] tensor. d in {64, 128}. has_v may carry MORJ_GEMM_FORCE_PAIR / MORJ_GEMM_FORCE_SINGLE.
 * rope: the RoPE table of morj_rope_table (rope_rows positions x d/2 (cos, sin) FP32 pairs), read at row
 * positions[row]; a position outside [0, rope_rows) sets the device error word (MORJ device code 0x301) and the row
 * is not written. rope, q_norm and k_norm 16-byte aligned. */
int morj_gemm_qkv_rope(const void* A, long long lda, const void* W, long long ldw, int M, int K, int hq, int hk,
                       int has_v, int d, const void* q_norm, const void* k_norm, const int* positions,
                       const void* rope, int rope_rows, const int* slots, float eps, void* q_out, void* k_pool,
                       void* v_pool, void* stream);

/* RoPE table by position (the reference's per-step cos / sin tables, lean_core.py:636-640, built once per model
 * and grown with the longest position seen): table[p][i] = (cos, sin)(p * inv_freq[i]) as FP32 pairs for
 * p < rows, i < half (half even). table 16-byte aligned, rows * half * 8 bytes. */
int morj_rope_table(const float* inv_freq, int half, int rows, void* table, void* stream);

/* Per row i < n: x[i] = bf16(embed[tokens[i]] * scale), or the feature row features[feature_row[i]] when
 * feature_row != NULL and feature_row[i] >= 0; then h[i] = bf16(rmsnorm(x[i]) * norm_w) (FP32 math). H % 8 == 0. */
int morj_embed_rmsnorm(const int* tokens, const int* feature_row, const void* features, const void* embed, int n,
                       int H, float scale, const void* norm_w, float eps, void* x_out, void* h_out, void* stream);

/* Per token i < n and head: RMSNorm over the head (q, k weighted; v unweighted), BF16 round, rotate-half RoPE at
 * angle positions[i] * inv_freq[j] (v: none); q heads go to q_out[i, hq, d], k and v heads to pool row
 * slots[i] of k_pool / v_pool ([slots, hk, d]). Column layout of qkv (leading dimension ld):
 * [hq q heads | hk k heads | hk v heads if has_v] x d; with has_v = 0 the v heads read the k columns.
 * hq or hk may be 0 (K/V-only and q-only calls). d in {64, 128, 256}. */
int morj_qkv_post(const void* qkv, long long ld, int n, int hq, int hk, int has_v, int d, const void* q_norm,
                  const void* k_norm, const int* positions, const float* inv_freq, const int* slots, float eps,
                  void* q_out, void* k_pool, void* v_pool, void* stream);

/* Work list for morj_tree_attention (host function, no device access): splits each segment's queries into tiles of
 * 128 / (hq / hk) queries and orders the tiles by the number of 64-key chunks they walk, longest first, from the host
 * copies of the attention call's segment tables (same meaning as there). Writes up to `cap` (segment, first query)
 * int pairs to work_host and returns the number of tiles (-1 if cap is too small). */
int morj_tree_attention_work(const int* qo_indptr_host, const int* kv_indptr_host, const int* kv_last_page_len_host,
                             int n_segments, int n_bidir, int hq, int hk, int page_size, int window, int* work_host,
                             int cap);

/* Tree-masked paged prefill attention. Segment s owns queries [qo_indptr[s], qo_indptr[s+1]) and the key list
 * pages kv_indices[kv_indptr[s] .. kv_indptr[s+1]) of page_size slots each (the last page holds
 * kv_last_page_len[s] slots, or is full when kv_last_page_len == NULL). Query j of a segment with q_len queries and
 * kv_len keys sees key t iff t <= kv_len - q_len + j (bottom-right causal) and, when window > 0,
 * t >= kv_len - q_len + j - (window - 1). The first n_bidir segments (image blocks) drop the causal bound and see
 * t >= kv_len - q_len + min(0, j - (window - 1)) (all keys when window <= 0).
 * q: [n_q, hq, d]; k_pool / v_pool: [pool_slots, hk, d]; out: [n_q, hq, d]; scores are scaled by sm_scale.
 * GQA: query head h reads kv head h / (hq / hk). d in {64, 128}. work: pairs from morj_tree_attention_work. */
int morj_tree_attention(const void* q, int n_q, const void* k_pool, const void* v_pool, int pool_slots, void* out,
                        const int* qo_indptr, const int* kv_indptr, const int* kv_indices,
                        const int* kv_last_page_len, int n_segments, int n_bidir, int hq, int hk, int d,
                        int page_size, int window, float sm_scale, const int* work, int n_work, void* stream);

/* Per row: o' = bf16(rmsnorm(o) * w_post); x = bf16(x + o'); h = bf16(rmsnorm(x) * w_pre). */
int morj_attn_epilogue(const void* o, void* x, void* h_out, const void* w_post, const void* w_pre, int n, int H,
                       float eps, void* stream);

/* Per row: d' = bf16(rmsnorm(d) * w_post); x = bf16(bf16(x + d') * scalar[0]); if has_next,
 * h = bf16(rmsnorm(x) * w_next). scalar is one BF16 value in device memory. h_out may alias x when !has_next. */
int morj_mlp_epilogue(const void* d, void* x, void* h_out, const void* w_post, const void* scalar,
                      const void* w_next, int n, int H, float eps, int has_next, void* stream);

/* dst[i, :] = src[rows[i], :] for i < n; width and leading dimensions in BF16 elements (multiples of 8). */
int morj_gather_rows(const void* src, long long ld_src, const int* rows, int n, int width, void* dst,
                     long long ld_dst, void* stream);

/* dst[rows[i], :] = src[i, :] for i < n (K/V pool head fill); width in BF16 elements (multiple of 8). */
int morj_scatter_rows(const void* src, long long ld_src, const int* rows, int n, int width, void* dst,
                      long long ld_dst, void* stream);

/* Label-restricted LM head. For each sequence j < n_seq: r = x[seq_row[j]], normed = bf16(rmsnorm(r) * norm_w);
 * logit_l = softcap * tanh((float(normed) . float(embed[label])) / softcap) over its labels
 * label_ids[label_indptr[j] .. label_indptr[j+1]) (at most 8192 per sequence); probs (FP32, same CSR layout) =
 * softmax over those logits. */
int morj_label_head(const void* x, long long ld_x, const int* seq_row, const int* label_indptr,
                    const int* label_ids, int n_seq, const void* norm_w, const void* embed, int H, float eps,
                    float softcap, float* probs, void* stream);

/* Reference-layout GeGLU (unfused path): out[i, j] = bf16(gelu_tanh(gu[i, j]) * gu[i, F + j]), gu: [n, 2F]. */
int morj_geglu(const void* gu, int n, int F, void* out, void* stream);

/* ---- tensor parallelism over peer memory (no counterpart in the reference, which runs one GPU per model; this
 * replaces the NCCL all-reduce after the row-parallel O and down projections of a T-way sharded model) ----------
 *
 * Rows are owned in blocks of 128: row block b belongs to rank b % world. Each rank's row-parallel GEMM stores its
 * BF16 partial rows in its own `part` buffer and counts the columns it wrote on the owner's per-block counter (an
 * atomic in the owner's memory); the owner's reduce kernel waits for all ranks' columns, reads the partial rows of
 * its blocks from every rank (NVLink loads from peer memory), sums them in rank order in FP32, rounds to BF16 (the
 * value an NCCL BF16 all-reduce gives for two ranks), applies the post-attention or post-MLP epilogue to its own
 * rows, and stores the new h rows (and, when asked, x rows) into every rank's buffers, counting rows on their
 * per-block counters. A wait kernel then holds the stream until every row block of h has arrived. Counters only
 * grow: the caller passes cumulative targets (site = one O or down reduction; after s sites every block's partial
 * counter reaches s * world * 4 * H and its row counter s * 128),
 * and blocks past a call's rows are padded by the reduce kernel so the targets hold for every block.
 * Every wait is bounded (2 s): on expiry the kernel records MORJ device code 0x104 / 0x105 and returns. */
#define MORJ_MAX_RANKS 8
typedef struct morj_peer {
  int world;       /* ranks (1..8) */
  int rank;        /* this rank */
  int max_blocks;  /* row blocks of 128 each buffer holds */
  int hidden;      /* H, columns of every exchanged row */
  void* part[MORJ_MAX_RANKS];                  /* rank r's partial rows, [max_blocks * 128, H] BF16 */
  void* x[MORJ_MAX_RANKS];                     /* rank r's residual rows, [max_blocks * 128, H] BF16 */
  void* h[MORJ_MAX_RANKS];                     /* rank r's normed rows, [max_blocks * 128, H] BF16 */
  unsigned long long* partials[MORJ_MAX_RANKS]; /* rank r's partial-column counters, [max_blocks] */
  unsigned long long* rows[MORJ_MAX_RANKS];     /* rank r's row counters, [max_blocks] */
} morj_peer_t;

/* CUDA IPC export of the device allocation holding `ptr` (handle: MORJ_IPC_HANDLE_BYTES bytes: the CUDA handle of
 * the allocation and ptr's offset in it), import on another process (peer access enabled; *ptr = the same byte),
 * and close of an imported pointer (with its handle). */
#define MORJ_IPC_HANDLE_BYTES 72
int morj_ipc_export(const void* ptr, void* handle);
int morj_ipc_import(const void* handle, void** ptr);
int morj_ipc_close(void* ptr, const void* handle);

/* Row-parallel GEMM: its BF16 partial rows C = A . B^T ([M, N], N = hidden, M <= max_blocks * 128) go to this
 * rank's part buffer, each tile counted on its row block owner's counter; the kernel is chosen per shape as for
 * morj_gemm_bf16. */
int morj_gemm_bf16_peer(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                        const morj_peer_t* peer, void* stream);

/* The owner's reduction of one site for rows [0, n): mode 0 = post-attention epilogue (w_a = post_attn,
 * w_b = pre_ff; morj_attn_epilogue's math), mode 1 = post-MLP epilogue (w_a = post_ff, scalar, w_b = next input
 * norm, has_next; morj_mlp_epilogue's math). x rows go to the peers only when push_x != 0. partial_target: the
 * cumulative partial count to wait for. */
int morj_peer_reduce(const morj_peer_t* peer, int mode, int n, const void* w_a, const void* scalar, const void* w_b,
                     float eps, int has_next, int push_x, unsigned long long partial_target, void* stream);

/* Hold the stream until every row block below n has reached row_target on this rank's row counters. */
int morj_peer_wait(const morj_peer_t* peer, int n, unsigned long long row_target, void* stream);

/* No counterpart in the reference. For callers that cannot allocate device memory (a process binding this C-ABI
 * from another language that owns only the buffers it passes in and may not call cudaMalloc itself): the one-rank
 * row-parallel projection and norm epilogue, C = A . B^T ([M, N] BF16, N = H) followed by morj_peer_reduce's
 * epilogue on every row (mode 0: post-attention, w_a = post_attn, w_b = pre_ff, h required; mode 1: post-MLP, w_a =
 * post_ff, scalar, w_b = next input norm, has_next). x is updated in place, h written. Its scratch (the C rows and
 * the block counters) is a fixed array inside the library, 8 MiB plus 16 KiB, held by every GPU that loads the
 * library until exit: M * N * 2 must not exceed 8 MiB (and M must not exceed 131072), larger calls are rejected
 * with MORJ_ERR_ARG. The first call on a device looks the array's address up (cudaGetSymbolAddress); make that
 * first call before any stream capture. The address is cached per device number for the process's life: after
 * cudaDeviceReset do not call it again in that process. h may be NULL for mode 1 with has_next = 0. Every call
 * shares the array: calls that overlap on the GPU race and must be ordered by the caller. Allocates nothing. */
int morj_gemm_norm_epilogue_noalloc(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                    int mode, void* x, void* h, const void* w_a, const void* scalar, const void* w_b,
                                    float eps, int has_next, void* stream);

/* ---- image path (reference VisionEncoder, lean_core.py:745-781: transformers' Gemma 4 vision tower and multimodal
 * embedder in BF16) ----------------------------------------------------------------------------------------------
 * The tower's projections, GeGLU MLP and residual epilogues use morj_gemm_bf16, morj_attn_epilogue and
 * morj_mlp_epilogue (layer scalar 1), its attention morj_tree_attention with one bidirectional segment per image.
 *
 * morj_vision_patch_prologue: pixels[i] = bf16(2 * bf16(pixels[i] - 0.5)) in place, n BF16 values (n % 8 == 0)
 * (Gemma4VisionPatchEmbedder's rescale).
 * morj_vision_position_add: x[r] += bf16(table[0][px] + table[1][py]) rounded to BF16, for n rows of H with patch
 * positions (px, py) = positions[2r], positions[2r+1]; padding patches (-1, -1) are left as they are; a position
 * outside [0, table_rows) sets the device error word (0x301). table: [2, table_rows, H] BF16.
 * morj_vision_head_epilogue: for n rows of the fused [q | k | v] projection (heads x d each, rows ld elements
 * apart): per head RMSNorm (q with q_norm, k with k_norm, v unweighted; BF16 output), then q and k get the 2-D rotary
 * embedding: head dims [0, d/2) rotated by the patch's x position, [d/2, d) by its y position, pairs (i, i + d/4)
 * within each half, angle position x inv_freq[i] (d/4 frequencies), cos/sin and every product rounded to BF16.
 * Writes q_out, k_out, v_out as [n, heads, d]. d in {64, 128}.
 * morj_vision_pool: out[c] = bf16(bf16(sum over r in cell_rows[cell_indptr[c] .. cell_indptr[c + 1]) of x[r] *
 * inv_k2) * scale) for n_cells cells (Gemma4VisionPooler's position-grid average and sqrt(hidden) scale).
 * morj_rmsnorm_rows: out[r] = bf16(x[r] * rsqrt(mean(x[r]^2) + eps) * w), w = 1 when NULL; H <= 16384. */
int morj_vision_patch_prologue(void* pixels, long long n, void* stream);
int morj_vision_position_add(void* x, const int* positions, const void* table, int table_rows, int n, int H,
                             void* stream);
int morj_vision_head_epilogue(const void* qkv, long long ld, int n, int heads, int d, const void* q_norm,
                              const void* k_norm, const int* positions, const float* inv_freq, float eps, void* q_out,
                              void* k_out, void* v_out, void* stream);
int morj_vision_pool(const void* x, int H, const int* cell_indptr, const int* cell_rows, int n_cells, float inv_k2,
                     float scale, void* out, void* stream);
int morj_rmsnorm_rows(const void* x, const void* w, int n, int H, float eps, void* out, void* stream);

/* ---- host planner (reference Tree, lean_core.py:34-231); host memory only, no CUDA ----------------------------
 *
 * morj_tree_build: the radix layout of n_seqs token sequences (tokens concatenated, seq_indptr[n_seqs + 1]); *tree
 * is an opaque handle, released with morj_tree_free. morj_tree_layout: sizes[3] = {nodes, path entries, node-path
 * entries}; with non-null arrays it also writes nodes[3 * n] (owner sequence, start depth, end depth; numbered by
 * start depth, ties by creation), offsets[n + 1], the per-sequence node paths (CSR: path_indptr[n_seqs + 1],
 * path_ids) and the per-node root paths (CSR: node_path_indptr[n + 1], node_path_ids). */
int morj_tree_build(const long long* tokens, const long long* seq_indptr, int n_seqs, void** tree);
int morj_tree_layout(const void* tree, long long* sizes, long long* nodes, long long* offsets, long long* path_indptr,
                     long long* path_ids, long long* node_path_indptr, long long* node_path_ids);
void morj_tree_free(void* tree);

/* Plan one pass over the nodes `compute` (in the caller's order) reading out `readout_seqs` (reference
 * Tree.plan_pass, same arguments): window, single_max, step_tokens, identity (slot = tree offset); prealloc: tree
 * offsets resident in slots 0.. (the shared head); initial_g/_s: per-kind slot tables of the previous pass
 * (num_tokens entries, -1 = none; both or neither); pinned_g/_s: offsets never freed; bidir: image-block node ids.
 * *plan is an opaque handle (morj_plan_free). Errors: MORJ_ERR_ARG (bad input, or a readout token is not computed
 * in the pass), MORJ_ERR_INTERNAL (a segment reads a token that has no slot).
 * morj_plan_blob: the plan as int64 values, in order:
 *   num_tokens, n_steps, cap_g, cap_s, n_readout; slot_of_g[num_tokens]; slot_of_s[num_tokens];
 *   readout (step, row)[n_readout];
 *   per step: n_segs, n_rows, n_bidir, n_kv_g, n_kv_s; segs (node, start depth, end depth)[n_segs]; own[n_rows]
 *   (tree offsets); positions[n_rows]; tokens[n_rows]; qo_indptr[n_segs + 1]; slots_g[n_rows]; slots_s[n_rows];
 *   kv_indptr_g[n_segs + 1]; kv_indices_g[n_kv_g]; kv_indptr_s[n_segs + 1]; kv_indices_s[n_kv_s].
 * The pointer stays valid until morj_plan_free. */
int morj_plan_pass(const void* tree, const long long* compute, int n_compute, const int* readout_seqs, int n_readout,
                   int window, long long single_max, long long step_tokens, int identity, const long long* prealloc,
                   long long n_prealloc, const long long* initial_g, const long long* initial_s,
                   const long long* pinned_g, long long n_pinned_g, const long long* pinned_s, long long n_pinned_s,
                   const long long* bidir, int n_bidir, void** plan);
int morj_plan_blob(const void* plan, const long long** data, long long* len);
void morj_plan_free(void* plan);

#ifdef __cplusplus
}
#endif

#endif /* MORJ_B200_H */
