/* xencb -- C ABI of the B200-native xenc Library read.
 *
 * One shared library (libxencb.so) with plain pointers and sizes: no torch, no C++ types. Every compute
 * entry point enqueues work on the CUDA stream `stream` (a cudaStream_t passed as void*; NULL = legacy
 * default stream), performs no host synchronisation and allocates no device memory: callers own every
 * buffer, including the scratch `workspace` whose size the matching *_workspace() query returns.
 *
 * Layouts (row-major, C order):
 *   rows        n_rows query tokens (the reference's [B, T] flattened), each reading one Library;
 *               row r reads Library  r / rows_per_lib.
 *   slots       a pool of n_pages pages; page p holds up to `page_rows` slot rows of d_s elements at
 *               slots + p * page_stride (elements). A Library is a table page_of[lib, c] -> page index
 *               with n_valid[lib, c] valid rows (the reference's mask, xenc/library.py:51-55).
 *   S           summary keys, float32 [n_lib, C, d_s] (xenc/library.py:69-74).
 *   weights     float32 in torch nn.Linear layout: [out_features, in_features]; output counts are multiples of 4.
 *               The projections run on the tcgen05 tensor cores (3xTF32) when in_features % 4 == 0 and the rows
 *               are 16-byte aligned, else on a CUDA-core fallback.
 *
 * Return value: XENCB_OK or an error code; xencb_last_error() gives the message of the last failing call on
 * the calling thread. XENCB_EINVAL is the reference's ValueError (bad shape / argument), the others are
 * runtime failures. Kernels never trap: a bounded wait that runs out sets a bit in the per-device status
 * word that xencb_device_status() returns.
 */
#ifndef XENCB_H_
#define XENCB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XENCB_ABI_VERSION 6

#if defined(__GNUC__)
#define XENCB_API __attribute__((visibility("default")))
#else
#define XENCB_API
#endif

/* status codes */
#define XENCB_OK 0
#define XENCB_EINVAL 1   /* invalid argument: maps to ValueError                         */
#define XENCB_ECUDA 2    /* CUDA runtime error (launch, attribute): RuntimeError         */
#define XENCB_ENOTSUP 3  /* valid but unsupported configuration: NotImplementedError    */

/* device status bits (xencb_device_status) */
#define XENCB_DEV_TIMEOUT 1u /* an mbarrier wait gave up after its time limit                  */
#define XENCB_DEV_CLAMPED 2u /* an n_valid entry exceeded page_rows and was clamped            */
#define XENCB_DEV_BADPAGE 4u /* a page_of entry was outside [0, n_pages); that chunk was skipped */
#define XENCB_DEV_BADROWS 8u /* a library_build row range was outside the row buffer; built empty */

/* element type codes */
#define XENCB_F32 0
#define XENCB_F16 1
#define XENCB_BF16 2

XENCB_API int xencb_abi_version(void);
XENCB_API const char* xencb_last_error(void);

/* Kernels launched (or captured into a CUDA graph) through this library in this process so far. No counterpart
 * in the reference: a diagnostic that lets a caller count the device work one call issues. */
XENCB_API unsigned long long xencb_launch_count(void);

/* Synchronises `stream`, returns the device status bits of the current device and clears them if `clear`. */
XENCB_API int xencb_device_status(void* stream, int clear, unsigned int* status_out);

/* ---------------------------------------------------------------------------------------------------------
 * Input projection: hn = rms_norm(h); q = L2(hn @ W_in^T + b_in); gate = sigmoid(hn . gate_w + gate_b).
 * Replaces xenc/injector.py:235-236 (rms_norm + itf_query, :54-58) and :266 (itf_gate, :61-65).
 *   flags    XENCB_PIN_RMS: multiply the input rows by 1/rms (rms_norm, no weight);
 *            XENCB_PIN_L2:  L2-normalise the output rows (x / (||x|| + 1e-6)).
 *            A full-rank A is one call with both flags; a low-rank A = Sequential(A1, A2) is a call with
 *            XENCB_PIN_RMS into a float32 [n_rows, rank] buffer, then one with XENCB_PIN_L2 over it.
 *   h        [n_rows, d_m] of h_dtype (the reference upcasts h to float32 first; so does this)
 *   w_in     [d_s, d_m] float32; b_in [d_s] or NULL; d_s % 4 == 0
 *   w_prep   NULL, or w_in prepared by xencb_weights_prep: the GEMM then runs as 3xF16 on the f16 tensor cores
 *            (fp32-faithful, see xencb_weights_prep; needs d_m % 8 == 0 and h 16-byte aligned, else the
 *            3xTF32 / SIMT path runs); w_in may then be NULL
 *   gate_w   [d_m] or NULL (then gate_out is not written); gate_b the scalar gate_b[pos[li]], or gate_b_dev a
 *            device pointer to it (when non-NULL it replaces gate_b: no host read of the parameter, so the call
 *            can be captured in a CUDA graph)
 *   sel_w    [n_cand, d_m] or NULL: LayerSelector logits z = hn @ sel_w^T + sel_b (xenc/selector.py:69-74)
 *   q_out    [n_rows, d_s] float32; gate_out [n_rows] or NULL; rstd_out [n_rows] or NULL (1/rms)
 *   z_out    [n_rows, n_cand] or NULL
 *   workspace at least xencb_project_in_workspace(n_rows, d_m, d_s) bytes, 256-byte aligned */
#define XENCB_PIN_RMS 1
#define XENCB_PIN_L2 2
XENCB_API size_t xencb_project_in_workspace(int64_t n_rows, int d_m, int d_s);
XENCB_API int xencb_project_in(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in,
                               const void* w_prep, const float* b_in, int d_s, int flags, const float* gate_w, float gate_b,
                               const float* gate_b_dev, const float* sel_w, const float* sel_b, int n_cand, float rms_eps, float* q_out,
                               float* gate_out, float* rstd_out, float* z_out, void* workspace,
                               size_t workspace_bytes, void* stream);

/* rms_norm alone (deltaskill.derive.rms_norm as called at xenc/injector.py:235): out = h * rsqrt(mean(h^2) + eps),
 * float32 out [n_rows, d_m]; for interfaces that are duck-typed objects (xenc/injector.py:55-56). */
XENCB_API int xencb_rms_norm(const void* h, int h_dtype, int64_t n_rows, int d_m, float eps, float* out,
                             void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Chunk routing. Replaces LibraryInjector.route (xenc/injector.py:220-229):
 *   logit[r, c] = (q[r] . S[lib(r), c]) * route_temp for c < n_chunks_of[lib] (else excluded);
 *   if 0 < top_k < n_chunks_of[lib]: keep the top_k logits, ties to the LOWER chunk index;
 *   softmax over the kept chunks.
 * Outputs: idx [n_rows, k_out] chunk ids sorted by (logit desc, index asc), -1 padded; wk [n_rows, k_out]
 * their weights (0 padded); w_dense [n_rows, C] the reference's w (zeros off the kept set) or NULL;
 * logit_out [n_rows, C] raw logits or NULL. k_out = xencb_route_k(top_k, C).
 * n_chunks_of may be NULL (every Library has C chunks). row_w [n_rows] may be NULL; a row with row_w == 0 (a
 * token whose LayerSelector weight for this layer is 0, xenc/selector.py:59-67, 106-110) gets idx -1 and wk 0,
 * so the read skips it, while its w_dense still holds the routing the reference reports. */
XENCB_API int xencb_route_k(int top_k, int n_chunks);
XENCB_API int xencb_route(const float* q, int64_t n_rows, int d_s, const float* S, int n_chunks, const int32_t* n_chunks_of,
                int64_t rows_per_lib, int64_t n_lib, float route_temp, int top_k, const float* row_w,
                int32_t* idx, float* wk, float* w_dense, float* logit_out, void* stream);

/* Decode form of xencb_project_in followed by xencb_route (xenc/injector.py:235-236, :54-58 and :220-229 in one
 * pass after the projection GEMM): each row's q is L2-normalised and routed in the same CTA, with the row's
 * summary keys fetched while the GEMM runs. Arguments as the two calls (the route's q is q_out); the outputs are
 * the same values (q bit for bit, the logits summed in the same order). Takes decode rows only: rows_per_lib < 64,
 * flags with XENCB_PIN_L2, d_s <= 6144 and (d_s + 2 * n_chunks) * 4 bytes <= 96 KiB; anything else returns
 * XENCB_ENOTSUP and launches nothing (use the two calls). Workspace: xencb_project_in_workspace bytes. */
XENCB_API int xencb_project_in_route(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in,
                                     const void* w_prep, const float* b_in, int d_s, int flags, const float* gate_w,
                                     float gate_b, const float* gate_b_dev, const float* sel_w, const float* sel_b,
                                     int n_cand, float rms_eps, float* q_out, float* gate_out, float* rstd_out,
                                     float* z_out, const float* S, int n_chunks, const int32_t* n_chunks_of,
                                     int64_t rows_per_lib, int64_t n_lib, float route_temp, int top_k,
                                     const float* row_w, int32_t* idx, float* wk, float* w_dense, float* logit_out,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* Decode form of xencb_project_in followed by xencb_route_lse (dense routing of a chunk shard for the sharded
 * read: xenc/injector.py:235-236, :54-58 and the routing softmax of :220-229 left unnormalised): the projection
 * GEMM, then per row q, its logits over every chunk and w_out = e^(l - max), header_out [n_rows, 4] =
 * (max, sum, 0, 0), the same values bit for bit as the two calls. The row's dot products are spread over up to
 * 32 CTAs. Takes what xencb_project_in_route takes (rows_per_lib < 64, flags with XENCB_PIN_L2, d_s <= 6144,
 * (d_s + 2 * n_chunks) * 4 bytes <= 96 KiB), else XENCB_ENOTSUP with nothing launched. Workspace:
 * xencb_project_in_workspace bytes. */
XENCB_API int xencb_project_in_route_lse(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in,
                                         const void* w_prep, const float* b_in, int d_s, int flags,
                                         const float* gate_w, float gate_b, const float* gate_b_dev, float rms_eps,
                                         float* q_out, float* gate_out, float* rstd_out, const float* S,
                                         int n_chunks, const int32_t* n_chunks_of, int64_t rows_per_lib,
                                         int64_t n_lib, float route_temp, float* w_out, float* header_out,
                                         void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Masked decode read over the routed chunks. Replaces the read of LibraryInjector._branch
 * (xenc/injector.py:239-245 and :263-265) for query rows that each read their own routed chunks:
 *   r[row] = sum_j wk[row, j] * read_c(q[row]),  c = idx[row, j] (skipped when c < 0 or wk == 0),
 *   read_c(q) = softmax_n(read_temp * q . k_cn) @ K_c   over the n_valid[lib, c] rows   (read_softmax != 0)
 *             = (sum_n (q . k_cn) k_cn) / sqrt(max(n_valid, 1))                         (read_softmax == 0)
 * K = V (tied) when vslots is NULL; otherwise vslots is the untied value pool (harvest="attn", xenc/library.py:
 * 46, 61-65; xenc/injector.py:211-218, 263-265) with the same dtype and page layout as slots: the scores use K,
 * the weighted sum uses V (f16 / bf16 slots and d_s % 16 == 0 only, else XENCB_ENOTSUP; this applies to
 * xencb_read_multi and xencb_read_prefill as well). slots_dtype XENCB_F16 / XENCB_BF16 / XENCB_F32;
 * accumulation is float32.
 * page_rows bounds n_valid (checked on the device: larger values are clamped and flagged). Slot pages and q
 * must be 16-byte aligned and d_s * sizeof(slot) a multiple of 16. The chunk read is split into row
 * ranges processed by a persistent, TMA-bulk-pipelined kernel and merged by log-sum-exp into r. */
XENCB_API size_t xencb_read_decode_workspace(int64_t n_rows, int k, int d_s, int page_rows, int slots_dtype);
XENCB_API int xencb_read_decode(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                      int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid,
                      int n_chunks, int64_t rows_per_lib, int64_t n_lib, const int32_t* idx, const float* wk, int k,
                      float read_temp, int read_softmax, float* r_out, void* workspace, size_t workspace_bytes,
                      void* stream);

/* The same read (xenc/injector.py:239-245, 263-265) planned for calls where many rows read nothing: rows whose
 * routing weights are all zero (the LayerSelector's row mask, xenc/selector.py:106-110, makes most tokens skip
 * most depths). Chunks are split into 128-row pieces and a one-CTA pass lists the pieces that hold rows, so the
 * live work spreads over every SM instead of over the few CTAs whose fixed share it falls in. Results match
 * xencb_read_decode within float32 rounding (the split sums are added in a different grouping). Tensor-core
 * (f16 / bf16, tied) reads of up to 65536 (row, chunk) pairs; other calls run the plan of xencb_read_decode. Workspace:
 * xencb_read_decode_sparse_workspace bytes. */
XENCB_API size_t xencb_read_decode_sparse_workspace(int64_t n_rows, int k, int d_s, int page_rows, int slots_dtype);
XENCB_API int xencb_read_decode_sparse(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots,
                                       int slots_dtype, int64_t n_pages, int64_t page_stride, int page_rows,
                                       const int32_t* page_of, const int32_t* n_valid, int n_chunks,
                                       int64_t rows_per_lib, int64_t n_lib, const int32_t* idx, const float* wk, int k,
                                       float read_temp, int read_softmax, float* r_out, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Attention diagnostics of LibraryInjector._branch.
 *
 * xencb_read_attn replaces record_attn (xenc/injector.py:259-260: last_attn[li] = aw[0, -1]): the route-weighted
 * slot attention of query row `row` (Library row / rows_per_lib), attn_out [n_chunks, page_rows] float32:
 *   attn[c, n] = wk[row, j] * softmax_n(read_temp * q[row] . k_cn)   for c = idx[row, j] and n < n_valid
 *                (read_softmax == 0: wk[row, j] * (q[row] . k_cn) / sqrt(max(n_valid, 1)))
 *   and 0 for chunks the row was not routed to and for rows past n_valid. Scores in float32 from the slots.
 * Arguments as xencb_read_decode (idx / wk as xencb_route writes them). */
XENCB_API int xencb_read_attn(const float* q, int64_t row, int d_s, const void* slots, int slots_dtype,
                              int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                              const int32_t* n_valid, int n_chunks, int64_t rows_per_lib, int64_t n_lib,
                              const int32_t* idx, const float* wk, int k, float read_temp, int read_softmax,
                              float* attn_out, void* stream);

/* xencb_read_forced replaces the force_attn override (xenc/injector.py:246-258) for one Library (page_of and
 * n_valid [n_chunks]): the given addressing fa [n_chunks, page_rows] float32 replaces the computed one for every
 * one of n_rows query rows,
 *   r_out[t] = s_t * sum_{c, n < n_valid[c]} fa[c, n] v_cn      (v = vslots when untied, else the slots)
 *   s_t = ||r0[t]|| / (||fa @ K|| + 1e-6) when norm_match (force_norm_match; r0 [n_rows, d_s] is the ordinary
 *   read, aw @ K), else 1; scale_out [n_rows] (or NULL) receives s_t. Workspace: xencb_read_forced_workspace
 *   bytes, 256-byte aligned. */
XENCB_API size_t xencb_read_forced_workspace(int n_chunks, int d_s);
XENCB_API int xencb_read_forced(const float* fa, int d_s, const void* slots, const void* vslots, int slots_dtype,
                                int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                                const int32_t* n_valid, int n_chunks, const float* r0, int64_t n_rows,
                                int norm_match, float* r_out, float* scale_out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Same read as xencb_read_decode, for callers that cannot allocate device memory at all: a host runtime that
 * owns every device byte through its own allocator and offers no way to request scratch, or a serving loop
 * that must not allocate (an allocation may synchronise the device). There is no counterpart of this entry
 * point in the reference; it exists for such callers of this library.
 * The scratch lives in a fixed device array inside libxencb.so, XENCB_NOALLOC_SCRATCH_BYTES bytes, which every
 * GPU that loads the library keeps until the process exits. A call whose scratch need
 * (xencb_read_decode_workspace) exceeds it returns XENCB_EINVAL and launches nothing. The first call on each
 * device looks up that array's device address (cudaGetSymbolAddress) with the device current; make that first
 * call before any stream capture. The address is kept for the life of the process: it does not survive
 * cudaDeviceReset or any other teardown of the device's primary context, after which this entry point must not
 * be called again in that process. All calls share the one array: calls on one device that overlap on the GPU
 * (issued to different streams) race and corrupt each other's results, so serialise them. Nothing in the
 * array needs to start at zero: the merge uses only words written earlier in the same call (it may load the
 * stale words of splits that hold no rows, and discards them). */
#define XENCB_NOALLOC_SCRATCH_BYTES (16u << 20)
XENCB_API int xencb_read_decode_noalloc(const float* q, int64_t n_rows, int d_s, const void* slots, int slots_dtype,
                                        int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                                        const int32_t* n_valid, int n_chunks, int64_t rows_per_lib, int64_t n_lib,
                                        const int32_t* idx, const float* wk, int k, float read_temp,
                                        int read_softmax, float* r_out, void* stream);

/* Many-query read over whole chunks (xenc/injector.py:239-265 with T > 1 query tokens per Library, the dense read
 * of BASELINE config 5): r[row] = sum_c w[row, c] * read(q[row], chunk c) with w [n_rows, n_chunks] float32 given
 * per (row, chunk) -- the routing softmax (dense or top-k with zeros), or unnormalised weights for a shard partial
 * (xencb_route_lse). Up to 8 query rows of a Library share every slot row read from HBM. Slots must be f16 or bf16
 * and d_s a multiple of 16 (<= 2560); other shapes return XENCB_ENOTSUP (use xencb_read_decode). Libraries,
 * pages and rows_per_lib as in xencb_read_decode; n_chunks_of [n_lib] may be NULL (all Libraries have
 * n_chunks chunks). Workspace: xencb_read_multi_workspace bytes, 256-byte aligned. */
XENCB_API size_t xencb_read_multi_workspace(int64_t n_rows, int64_t rows_per_lib, int n_chunks, int d_s, int page_rows,
                                            int slots_dtype);
XENCB_API int xencb_read_multi(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                               int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                               const int32_t* n_valid, int n_chunks, const int32_t* n_chunks_of, int64_t rows_per_lib,
                               int64_t n_lib, const float* w, float read_temp, int read_softmax, float* r_out,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Prefill (registration) read on the tensor cores: the same result as xencb_read_multi, computed as two tcgen05
 * GEMMs for many query tokens per Library (T = 2048 tokens per document, every chunk read).
 * w [n_rows, n_chunks] float32 as in xencb_read_multi. Requirements: f16 slots, d_s a multiple of 64,
 * page_rows <= 512, a dense pool (page_stride == page_rows * d_s); rows of a page past n_valid must be finite
 * (they are multiplied by 0). Other shapes return XENCB_ENOTSUP. q is rounded to f16 for the score product.
 * Workspace: xencb_read_prefill_workspace bytes (q in f16 + the f16 weights P [n_rows, n_chunks * round_up(page_rows, 64)]). */
XENCB_API size_t xencb_read_prefill_workspace(int64_t n_rows, int n_chunks, int d_s, int page_rows);
XENCB_API int xencb_read_prefill(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                                 int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                                 const int32_t* n_valid, int n_chunks, const int32_t* n_chunks_of,
                                 int64_t rows_per_lib, int64_t n_lib, const float* w, float read_temp,
                                 int read_softmax, float* r_out, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Dense routing of one chunk shard of a Library (the routing softmax of xenc/injector.py:220-229 with top_k = 0,
 * regrouped by shard): w_out [n_rows, n_chunks] = e^(l_c - max_c l_c) with l = route_temp * q . S_c, and
 * header_out [n_rows, 4] = (max_c l_c, sum_c e^(l_c - max), 0, 0). Feeding w_out to xencb_read_multi gives the
 * shard's accumulator A = sum_c e^(l_c - max) r_c; (header, A) is the shard's partial. */
XENCB_API int xencb_route_lse(const float* q, int64_t n_rows, int d_s, const float* S, int n_chunks,
                              const int32_t* n_chunks_of, int64_t rows_per_lib, int64_t n_lib, float route_temp,
                              float* w_out, float* header_out, void* stream);

/* Combines the partials of n_shards chunk shards into the read of the whole Library:
 * parts [n_shards][n_rows * 4 + n_rows * d_s] holds per shard the headers of xencb_route_lse then the
 * accumulators of xencb_read_multi (the layout an all-gather of each shard's block produces);
 * r = sum_g e^(max_g - M) A_g / sum_g e^(max_g - M) sum_g with M the largest max_g. */
XENCB_API int xencb_shard_merge(const float* parts, int n_shards, int64_t n_rows, int d_s, float* r_out, void* stream);

/* Exchange of the partial blocks over NVLink peer memory, in place of the all-gather before xencb_shard_merge
 * (one process per GPU, every rank on its own GPU of one node). Each rank allocates an exchange buffer of
 * xencb_exch_bytes(world, per) bytes (per = n_rows * (4 + d_s) floats, the block of xencb_shard_merge) with
 * xencb_exch_alloc, which also returns its CUDA IPC handle (64 bytes); the ranks swap handles on the host and open
 * each other's buffers with xencb_exch_open. A step is then
 *   xencb_shard_push(block, ...)          this rank's block into slot `rank` of every rank's buffer (plain peer
 *                                         stores), and that slot's flag raised to the step's epoch;
 *   xencb_shard_merge_wait(own buffer, ...) waits for every rank's flag, then the merge of xencb_shard_merge.
 * peers_dev: device array [world] of uint64 buffer addresses (this rank's own buffer at index `rank`, the opened
 * peer mappings elsewhere). state: 3 uint32 of device memory, zero before the first push, kept across steps (the
 * epochs; a CUDA graph of a step can be replayed). Blocks of consecutive steps alternate between two halves of
 * the buffer, so a rank one step ahead never overwrites a block that is being merged. A flag that does not
 * arrive within about 1.5 s sets XENCB_DEV_TIMEOUT. xencb_exch_close unmaps a peer buffer, xencb_exch_free frees
 * the rank's own. world <= 64. */
XENCB_API size_t xencb_exch_bytes(int world, int64_t per);
XENCB_API int xencb_exch_alloc(size_t bytes, void** ptr, void* handle_out);
XENCB_API int xencb_exch_open(const void* handle, void** peer_ptr);
XENCB_API int xencb_exch_close(void* peer_ptr);
XENCB_API int xencb_exch_free(void* ptr);
XENCB_API int xencb_shard_push(const float* block, int64_t per, const void* peers_dev, int world, int rank,
                               uint32_t* state, void* stream);
XENCB_API int xencb_shard_merge_wait(const void* exch, int world, int64_t n_rows, int d_s, const uint32_t* state,
                                     float* r_out, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Output projection and injection epilogue. Replaces xenc/injector.py:266-267 (gain_scale * gain * gate *
 * itf_write(r), :74-77), LayerSelector.apply (xenc/selector.py:95-110) and the hook arithmetic
 * (xenc/injector.py:185-197: delta.to(h.dtype), position mask, mag term, h + delta):
 *   d        = scale * gate[row] * (r @ W_out^T + b_out)                 (gate NULL -> 1)
 *   if sel_w: d = sel_w[row] * exp(log_alpha) * d / (||d|| / (||h|| + 1e-6) + 1e-6)
 *   log_scale_dev (device float or NULL): the scale is multiplied by exp(*log_scale_dev) (the interface's
 *   log_gain[pos] read on the device); log_alpha_dev (device float or NULL) replaces log_alpha. Both keep the
 *   call free of host reads of parameters, so it can be captured in a CUDA graph.
 *   d       *= pos_mask[row]                                              (pos_mask NULL -> 1)
 *   delta_out = d in h_dtype (or NULL); h_out = h + delta_out in h_dtype (or NULL; may alias h);
 *   rel_out[row] = ||delta_out|| / (||h|| + 1e-6)                         (or NULL)
 *   h        [n_rows, d_m] of h_dtype; r [n_rows, d_s] float32; w_out [d_m, d_s]; b_out [d_m] or NULL;
 *            d_m % 4 == 0. w_prep: NULL or w_out prepared by xencb_weights_prep (as for xencb_project_in). */
XENCB_API size_t xencb_project_out_workspace(int64_t n_rows, int d_s, int d_m);
XENCB_API int xencb_project_out(const float* r, int64_t n_rows, int d_s, const float* w_out, const void* w_prep,
                                const float* b_out, int d_m,
                      float scale, const float* log_scale_dev, const float* gate, const float* sel_w, float log_alpha,
                      const float* log_alpha_dev, const float* pos_mask,
                      const void* h, int h_dtype, void* delta_out, void* h_out, float* rel_out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * LayerSelector weights from logits. Replaces LayerSelector._weights_from_logits (xenc/selector.py:59-67),
 * forward value: top-k of z (ties to the lower index), softmax over the kept (or 1/k when
 * straight_through), zeros elsewhere. z, w_out: [n_rows, n_cand] float32, n_cand <= 32. */
XENCB_API int xencb_selector_weights(const float* z, int64_t n_rows, int n_cand, int k, int straight_through, float* w_out,
                           void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * LayerSelector logits. Replaces LayerSelector.compute (xenc/selector.py:69-74): z = x @ u_w^T + u_b, with
 * x = rms_norm(h) when `rms` != 0 (the recompute at the first candidate layer, :98-101) or x = h as given
 * (an explicit compute(hn0)). h [n_rows, d_m] of h_dtype; u_w [n_cand, d_m]; u_b [n_cand] or NULL. */
XENCB_API int xencb_selector_logits(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* u_w,
                                    const float* u_b, int n_cand, int rms, float rms_eps, float* z_out, void* stream);

/* LayerSelector.apply once the weights exist (xenc/selector.py:106-110), for a delta computed elsewhere:
 *   out = w[row, pos] * exp(log_alpha) * d / (||d|| / (||h|| + 1e-6) + 1e-6),  d = float32(delta)
 * delta [n_rows, d] of delta_dtype; h [n_rows, d] of h_dtype; w [n_rows, n_cand] float32; out like delta. */
XENCB_API int xencb_selector_apply(const void* delta, int delta_dtype, const void* h, int h_dtype, int64_t n_rows,
                                   int d, const float* w, int n_cand, int pos, float log_alpha, void* out,
                                   void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Summary keys on the device. Replaces Library._summaries (xenc/library.py:69-74):
 *   S[lib, c] = L2(mean of the n_valid[lib, c] rows of page page_of[lib, c]) (zero rows give S = 0). */
XENCB_API int xencb_summaries(const void* slots, int slots_dtype, int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                    const int32_t* n_valid, int64_t n_lib, int n_chunks, int d_s, float* S_out, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Library build on the device, for one depth of one or several Libraries. Replaces the per-chunk host loop of
 * Library.__init__ (xenc/library.py:47-67) and Library._summaries (xenc/library.py:69-74):
 *   rows       [n_rows_total, d_s] of rows_dtype: the doc cache's rows of every chunk, concatenated in chunk order
 *   row_start  [n_chunks + 1] int64 (device): chunk c is rows [row_start[c], row_start[c + 1])
 *   mu         [d_s] float32 or NULL: centering, K = L2(K - mu) on the chunk's rows (xenc/library.py:56-58)
 * Page page_of[c] of `slots` (slots_dtype, page_rows x d_s, page_stride elements apart) receives the chunk's
 * rows, then zeros up to page_rows; n_valid_out[c] = the row count (NULL: not written); S_out[c] = L2(mean of
 * the chunk's rows) in float32, computed before the rows are rounded to slots_dtype (NULL: not written).
 * d_s % 8 == 0; rows, slots and page_stride * element size 16-byte aligned. On the device a row range outside
 * [0, n_rows_total] builds an empty chunk (XENCB_DEV_BADROWS) and a chunk longer than page_rows is cut
 * (XENCB_DEV_CLAMPED). The result is deterministic (fixed summation order). */
XENCB_API size_t xencb_library_build_workspace(int n_chunks, int d_s, int page_rows);
XENCB_API int xencb_library_build(const void* rows, int rows_dtype, int64_t n_rows_total, const int64_t* row_start,
                                  int n_chunks, int d_s, const float* mu, void* slots, int slots_dtype,
                                  int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                                  int32_t* n_valid_out, float* S_out, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * D8 top-k slot selection and read (xenc/topk_read.py). Slot s of a Library is row s % page_rows of its chunk
 * s / page_rows (the residual Library's padded [C, N] slot grid, flattened as the reference's Kf[idx]).
 *
 * xencb_select_scores replaces TopKSelector.head_scores + pool_scores (xenc/topk_read.py:215-239):
 *   scores[r, s] = pool_h pool_t (q[r, t, h, :] . keys[lib(r), s, h / (n_q / n_kv), :])
 *   q [n_rows, T, n_q, hd] float32 (the reader's pre-RoPE queries at the selection layer, T positions);
 *   keys per Library [n_chunks * page_rows, n_kv * hd], XENCB_F32 or XENCB_F16, keys_lib_stride elements apart;
 *   query_pool 0 = max over T (T = 1 for query "last"), 1 = mean; head_pool 0 = max, 1 = mean;
 *   slots at or past n_valid of their chunk, or in chunks past n_chunks_of[lib], score -inf.
 * xencb_select_topk replaces sc.topk(k) (xenc/topk_read.py:251-254): per row the k largest scores, sorted by
 *   score (descending), ties to the lower slot; idx_out [n_rows, k] int32, score_out [n_rows, k] (or NULL).
 *   k <= 2048 and k <= n_slots.
 * xencb_topk_read replaces TopKLibraryInjector._branch's read (xenc/topk_read.py:392-413):
 *   a = q . K[idx] over the k slots of the row's index set, softmax(a * read_temp) or a / sqrt(k), r = a @ V[idx]
 *   (V = vslots when not NULL, else K). Rows [b * n_rows / n_sets, (b + 1) * n_rows / n_sets) use idx[b] and
 *   Library b when n_lib > 1 (else Library 0). attn_out [n_rows, k] receives a (NULL: not written). */
XENCB_API int xencb_select_scores(const float* q, int64_t n_rows, int T, int n_q, int n_kv, int hd, const void* keys,
                                  int keys_dtype, int64_t keys_lib_stride, int page_rows, int n_chunks,
                                  const int32_t* n_valid, const int32_t* n_chunks_of, int64_t rows_per_lib,
                                  int64_t n_lib, int query_pool, int head_pool, float* scores_out, void* stream);
XENCB_API int xencb_select_topk(const float* scores, int64_t n_rows, int n_slots, int k, int32_t* idx_out,
                                float* score_out, void* stream);
XENCB_API int xencb_topk_read(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots,
                              int slots_dtype, int64_t n_pages, int64_t page_stride, int page_rows,
                              const int32_t* page_of, int n_chunks, int64_t n_lib, const int32_t* idx, int n_sets,
                              int k, float read_temp, int read_softmax, float* r_out, float* attn_out, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Weight preparation for the 3xF16 projection GEMM (done once per weight tensor, e.g. when an interface is
 * loaded): w [n, k] float32 -> prep = a 256-byte head (max |w|, 1/s) followed by the f16 pair hi, lo of
 * w * s, s = 2^e with max|w| * s in [2^14, 2^15), in 128 x 64 tiles (per 128-row band and 64-column block, the
 * hi tile then the lo tile, 32 KiB, bands outer; zeros past n and k), so that the GEMM reads each CTA's share
 * of the weight as one contiguous run. hi + lo keeps ~22 mantissa bits, and the GEMM sums hi*hi + hi*lo +
 * lo*hi (the relative error of the 3xTF32 product). k % 8 == 0; prep 256-byte aligned, at least
 * xencb_weights_prep_bytes(n, k) bytes (4 bytes per weight with n rounded up to 128 and k to 64, + 256). */
XENCB_API size_t xencb_weights_prep_bytes(int n, int k);
XENCB_API int xencb_weights_prep(const float* w, int n, int k, void* prep, size_t prep_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Failure-detection self-test of the bounded waits every pipelined kernel uses: one thread waits, with a limit
 * of limit_cycles SM cycles (the kernels use 3e9), on an mbarrier phase that nothing completes. The wait gives
 * up, raises XENCB_DEV_TIMEOUT in the device status word and the kernel returns; *result (device int, or NULL)
 * becomes 0. The context stays usable. */
XENCB_API int xencb_wait_selftest(long long limit_cycles, int* result, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Instrumentation for kernel timing with CUDA events: the next xencb_read_decode call on this host thread records
 * `before` and `after` (cudaEvent_t created by the caller, timing enabled; either may be NULL) on its stream
 * immediately before and after its main read kernel, so their interval excludes the merge launch. One-shot:
 * the call consumes the pair. No reference counterpart (measurement only). */
XENCB_API int xencb_read_kernel_events(void* before, void* after);

#ifdef __cplusplus
}
#endif

#endif /* XENCB_H_ */
