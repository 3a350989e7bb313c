/*
 * cpu_attention_b200.h -- the C ABI of the B200 (sm_100a) build of cpu-attention.
 *
 * One shared object (libca_b200.so) replaces the reference's per-ISA-tier Mojo
 * extensions (`cpu_attention/_kernel.py:52-84` loads one `_C_<tier>.so`). Its
 * entries take plain device pointers, sizes and element strides; nothing in the
 * signatures is a torch type, so any host language binds them (ctypes, cgo,
 * JNI, N-API). Every compute entry is asynchronous on the caller's CUDA stream.
 *
 * Return convention (restates `_C.mojo:1-8`: "returns None for anything it does
 * not take"): 0 = done; a negative CA_E* code = declined, nothing was launched,
 * and the caller raises the precise error (the Python layer maps each code to
 * the reference's ValueError / NotImplementedError text).
 *
 * Value errors that only the device can see (a cache_seqlens entry past the
 * page table's capacity, a page-table entry or slot past the cache) never cause
 * an out-of-bounds access: the kernels skip the offending work and OR a
 * CA_STATUS_* bit into a status word in the workspace, read back with
 * ca_status().
 *
 * dtype codes follow `_kernel.py:17` (DTYPES = {float32: 0, bfloat16: 1}).
 */
#ifndef CPU_ATTENTION_B200_H
#define CPU_ATTENTION_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CA_API __attribute__((visibility("default")))
#else
#define CA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- codes ------------------------------------------------------------ */
#define CA_DTYPE_F32 0
#define CA_DTYPE_BF16 1

#define CA_OK 0
#define CA_EDTYPE -1        /* dtype not fp32/bf16, or operands disagree      */
#define CA_EHEADDIM -2      /* head_dim not 32/64/128                          */
#define CA_EPAGE -3         /* page size not a positive multiple of 16         */
#define CA_ESHAPE -4        /* sizes disagree (batch, heads, tokens, tables)   */
#define CA_ELAYOUT -5       /* a stride/alignment the kernel cannot read       */
#define CA_ENULL -6         /* a required pointer is NULL                      */
#define CA_EWORKSPACE -7    /* workspace missing or too small                  */
#define CA_ECUDA -8         /* a CUDA runtime call failed (ca_last_cuda_error) */
#define CA_EUNSUPPORTED -9  /* a shape this build does not implement           */
#define CA_ESCRATCH -10     /* beyond ca_decode_noalloc's static scratch        */

/* status bits written by the device into the workspace (ca_status) */
#define CA_STATUS_LENS 1    /* cache_seqlens (+ the appended token) past W*page */
#define CA_STATUS_TABLE 2   /* a page-table entry outside [0, num_blocks)      */
#define CA_STATUS_SLOT 4    /* a slot_mapping entry >= num_blocks * page       */
#define CA_STATUS_TIMEOUT 8 /* a bounded device wait gave up                   */

/* ---- reshape_and_cache -------------------------------------------------
 * Replaces `_C.store(rt, key, value, k_cache, v_cache, slots)` (`_C.mojo:174-213`)
 * behind `cache.py:13-25` `reshape_and_cache`.
 * key/value: [num_tokens, heads, head_dim] with heads and dims contiguous and
 *   `token_stride` elements between tokens (both share it, `_C.mojo:198`).
 * k_cache/v_cache: [num_blocks, heads, page, head_dim] contiguous, the reference's
 *   in-page layout (`paged_attn.mojo:58-131`): K of token t, dim d at element
 *   ((d>>1)*page + t)*2 + (d&1) (bf16) or d*page + t (fp32) of its (block, head)
 *   page; V at t*head_dim + d.
 * slots: int64 [num_tokens]; token i goes to page slots[i] / page, position
 *   slots[i] % page; a negative slot skips the token (`paged_attn.mojo:155-158`).
 *   Slots >= num_blocks*page are skipped and flagged (CA_STATUS_SLOT) in
 *   `status` when it is non-NULL (a device int32).
 */
CA_API int ca_store(const void* key, const void* value, int64_t token_stride,
             void* k_cache, void* v_cache, int64_t num_blocks,
             const int64_t* slots, int64_t num_tokens, int64_t heads,
             int64_t head_dim, int64_t page, int dtype, int32_t* status,
             void* stream);

/* ---- paged decode (flash_attn_with_kvcache, one query token) -----------
 * Replaces `_C.decode(rt, q, k_cache, v_cache, k, v, slots, lens, page_table,
 * scale, dst)` (`_C.mojo:87-171`), called by `flash_attn_interface.py:150-159`
 * and by an engine directly (`examples/ops.py:19-31`).
 * q: [batch, heads, head_dim] rows, heads and dims contiguous, `q_stride`
 *   elements between sequences (any token stride: fused projections).
 * k_new/v_new: NULL (cross-attention: no store), or the new token's K/V, same
 *   row layout with `kv_stride` elements between sequences.
 * slots: NULL = append each new token at position lens[i] through the page
 *   table (`paged_attn.mojo:162-168`), and attend lens[i] + 1 keys; non-NULL =
 *   store at slots[i] (int64, negative skips) and attend lens[i] keys
 *   (`_C.mojo:100-103`, `paged_attn.mojo:723-725`).
 * lens: int32 [batch]; page_table: int32 [batch, table_width] contiguous.
 * out: [batch, heads, head_dim] contiguous (`_C.mojo:154-160`).
 * softmax_scale: NaN selects the default head_dim ** -0.5 (`_C.mojo:168`).
 * workspace: device memory of at least ca_decode_workspace_bytes() bytes,
 *   zero-filled once before its first use; calls that overlap in time on the
 *   device must not share one. A row that sees no key is exactly 0
 *   (`paged_attn.mojo:297-310`).
 */
CA_API size_t ca_decode_workspace_bytes(int64_t batch, int64_t heads, int64_t head_dim,
                                 int64_t page, int dtype, int device);

CA_API int ca_decode(const void* q, int64_t q_stride, void* k_cache, void* v_cache,
              int64_t num_blocks, const void* k_new, const void* v_new,
              int64_t kv_stride, const int64_t* slots, const int32_t* lens,
              const int32_t* page_table, int64_t table_width, void* out,
              int64_t batch, int64_t heads, int64_t head_dim, int64_t page,
              int dtype, float softmax_scale, void* workspace,
              size_t workspace_bytes, void* stream);

/* ---- decode with a several-token append, in one launch ---------------------
 * Replaces the reference's two-step path for k/v holding several new tokens
 * per sequence (`flash_attn_interface.py:109-117`: the tokens are stored at
 * cache_seqlens + j by `reshape_and_cache`, then `_C.decode` attends the grown
 * cache). Here the decode launch itself writes
 * the tokens (the warp that streams a page holding new tokens patches them in
 * and writes them to the cache) and attends lens[i] + n_new keys.
 * k_new/v_new: token j of sequence i at element i * kv_stride +
 *   j * kv_token_stride (+ head * head_dim + dim); kv_token_stride >=
 *   heads * head_dim and kv_stride >= n_new * kv_token_stride.
 * The other arguments are ca_decode's with slots = NULL. n_new = 1 is
 * ca_decode's fused one-token append.
 */
CA_API int ca_decode_append(const void* q, int64_t q_stride, void* k_cache,
              void* v_cache, int64_t num_blocks, const void* k_new,
              const void* v_new, int64_t kv_stride, int64_t kv_token_stride,
              int64_t n_new, const int32_t* lens, const int32_t* page_table,
              int64_t table_width, void* out, int64_t batch, int64_t heads,
              int64_t head_dim, int64_t page, int dtype, float softmax_scale,
              void* workspace, size_t workspace_bytes, void* stream);

/* ---- the general decode entry: grouped heads, log-sum-exp -----------------
 * ca_decode and ca_decode_append in one entry, with two capabilities the
 * reference declines (`flash_attn_interface.py:87-96`, `:144-145`):
 * kv_heads: the heads of the caches and of k_new/v_new; heads % kv_heads == 0
 *   and query head h attends KV head h / (heads / kv_heads) (GQA; MQA at
 *   kv_heads = 1). kv_heads == heads is ca_decode.
 * lse: NULL, or float32 [batch, heads]: each row's log-sum-exp,
 *   ln(sum_t exp(scale * q . k_t)), -inf for a row that sees no key
 *   (flash-attn's softmax_lse).
 * n_new: 0 (k_new/v_new NULL: no new tokens), 1 (stored at slots[i], or
 *   appended at lens[i] when slots is NULL) or more (appended at lens[i],
 *   kv_token_stride elements apart; slots NULL).
 * The workspace is ca_decode_workspace_bytes(batch, heads, ...) long.
 */
CA_API int ca_decode_ex(const void* q, int64_t q_stride, void* k_cache,
              void* v_cache, int64_t num_blocks, const void* k_new,
              const void* v_new, int64_t kv_stride, int64_t kv_token_stride,
              int64_t n_new, const int64_t* slots, const int32_t* lens,
              const int32_t* page_table, int64_t table_width, void* out,
              float* lse, int64_t batch, int64_t heads, int64_t kv_heads,
              int64_t head_dim, int64_t page, int dtype, float softmax_scale,
              void* workspace, size_t workspace_bytes, void* stream);

/* ---- paged decode without allocation -----------------------------------
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory (an engine that reserves all GPU memory up front and
 * forbids later allocations; a plugin interface that passes only input and
 * output buffers). Same arguments and result as ca_decode, minus the
 * workspace: it runs ca_decode with a static device array of the library as
 * the workspace and allocates nothing.
 * Limits: batch * heads <= 65536 and at most 160 SMs, else CA_ESCRATCH and
 *   nothing is launched. The array (about 5.3 MiB) stays resident on every
 *   GPU that loads the library until the process exits.
 * Every call shares the array: calls that overlap on the GPU race; order them.
 *   Device-found value errors are skipped but not reported (validate on the
 *   host). The first call on a device looks up the array's address; make it
 *   before any stream capture. The address is kept for the life of the
 *   process: a cudaDeviceReset after that first call is not supported.
 */
CA_API int ca_decode_noalloc(const void* q, int64_t q_stride, void* k_cache,
              void* v_cache, int64_t num_blocks, const void* k_new,
              const void* v_new, int64_t kv_stride, const int64_t* slots,
              const int32_t* lens, const int32_t* page_table,
              int64_t table_width, void* out, int64_t batch, int64_t heads,
              int64_t head_dim, int64_t page, int dtype, float softmax_scale,
              void* stream);

/* ---- dense prefill (flash_attn_func) ------------------------------------
 * Replaces `_C.flash(rt, q, k, v, scale, causal, ws, ws_bytes)`
 * (`_C.mojo:232-316`) behind `flash_attn_interface.py:168-193`.
 * q: [batch, seq_q, heads, head_dim]; k/v: [batch, seq_k, heads, head_dim];
 *   strides in elements (batch, token, head); the dim stride must be 1
 *   (`_C.mojo:263`). out: [batch, seq_q, heads, head_dim] contiguous.
 * causal: bottom-right aligned, row i sees keys j <= i + seq_k - seq_q; a row
 *   that sees no key is exactly 0 (`flash_attn.mojo:127-183`).
 * softmax_scale: NaN selects head_dim ** -0.5.
 * status: NULL, or a device int32 that receives CA_STATUS_TIMEOUT if a
 *   bounded device wait gives up.
 * bf16 runs on the tensor cores (tcgen05, TMA-fed) whenever TMA can describe
 * q/k/v (16-byte aligned base and strides); fp32 and other bf16 layouts run on
 * a CUDA-core kernel.
 */
CA_API int ca_flash(const void* q, const void* k, const void* v, void* out,
             int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads,
             int64_t head_dim, const int64_t q_strides[3],
             const int64_t k_strides[3], const int64_t v_strides[3],
             float softmax_scale, int causal, int dtype, int32_t* status,
             void* stream);

/* ---- the general prefill entry: grouped heads, log-sum-exp, varlen -------
 * ca_flash with three capabilities the reference declines
 * (`flash_attn_interface.py:144-145`, `:215-218`):
 * kv_heads: k/v's heads; heads % kv_heads == 0 and query head h attends KV
 *   head h / (heads / kv_heads) (GQA; MQA at kv_heads = 1).
 * lse: NULL, or float32 rows of log-sum-exp, ln(sum_j exp(scale * q . k_j)),
 *   -inf for a row that sees no key: [batch, heads, seq_q] (dense) or
 *   [heads, total_q] (varlen) -- flash-attn's softmax_lse.
 * cu_seqlens_q / cu_seqlens_k: NULL (dense), or device int32 [batch + 1]
 *   (varlen, flash_attn_varlen_func): sequence b's queries are tokens
 *   [cu_seqlens_q[b], cu_seqlens_q[b + 1]) of q [total_q, heads, head_dim] and
 *   its keys tokens [cu_seqlens_k[b], cu_seqlens_k[b + 1]) of k/v
 *   [total_k, kv_heads, head_dim]; seq_q / seq_k are then the largest
 *   sequence lengths (no sequence may exceed them), the strides' batch entry
 *   is ignored, out is [total_q, heads, head_dim] and causal masks per
 *   sequence (bottom-right). total_q / total_k are ignored when dense.
 */
CA_API int ca_flash_ex(const void* q, const void* k, const void* v, void* out,
             float* lse, int64_t batch, int64_t seq_q, int64_t seq_k,
             int64_t heads, int64_t kv_heads, int64_t head_dim,
             const int64_t q_strides[3], const int64_t k_strides[3],
             const int64_t v_strides[3], const int32_t* cu_seqlens_q,
             const int32_t* cu_seqlens_k, int64_t total_q, int64_t total_k,
             float softmax_scale, int causal, int dtype, int32_t* status,
             void* stream);

/* ---- runtime ------------------------------------------------------------ */
/* The status word of a decode workspace (ORed CA_STATUS_* bits since the last
 * reset); synchronises `stream`. reset != 0 clears it; when the word holds
 * CA_STATUS_TIMEOUT it also clears what a decode that gave up leaves behind
 * (its task counter and the tickets of its (sequence, head) items), so the
 * workspace serves the next call again. Returns < 0 on a CUDA error. */
CA_API int ca_status(void* workspace, int reset, void* stream);

/* The limit of each bounded device wait of the decode kernels from the next
 * call on (process-wide), in nanoseconds; 0 restores the default of 2 s. No
 * counterpart in the reference: it exists so that failure handling can be
 * tested (a wait that runs out sets CA_STATUS_TIMEOUT and the kernel returns)
 * without faulting or hanging a GPU. */
CA_API void ca_set_wait_limit_ns(uint64_t ns);

/* The last CUDA error string seen by this library on this host thread. */
CA_API const char* ca_last_cuda_error(void);

/* "sm_100a" plus the build's CUDA version, for diagnostics (the counterpart of
 * `_C.tier()`, `_C.mojo:347-349`). */
CA_API const char* ca_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* CPU_ATTENTION_B200_H */
