/* libjeffb200: the C ABI of the B200-native decision hot path (sm_100a).
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t (as void*), launches its kernels on that
 * stream and returns a status (JB_OK or a negative code; jb_last_error() gives the message). No entry point
 * allocates device memory or synchronises, so all of them can be recorded into a CUDA graph; buffers belong to the
 * caller. bf16 tensors are passed as uint16_t* (bfloat16 bit patterns), row-major and contiguous unless a leading
 * dimension is given.
 *
 * Each declaration names the reference interface it replaces (firelex/jeff, paths under
 * runtime/python/src/jeff_runtime/engine/). The prefix pool geometry is the reference's (prefix_pool.py:1-40):
 * pages of page_bytes bytes; state[page][head slot][128][128] fp32, conv[page][layer slot][3][6144] bf16,
 * kv[page][attn layer][K|V][32 tokens][2 heads][256] bf16; block tables int32 [row][state pages | conv pages |
 * key/value pages]. */
#ifndef JEFFB200_H
#define JEFFB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JB_OK 0
#define JB_EINVAL (-1)   /* an argument the kernels cannot take (checked before any launch) */
#define JB_ECUDA (-2)    /* a CUDA runtime error */
#define JB_ETIMEOUT (-3) /* a device-side bounded wait gave up (see jb_device_status) */
#define JB_DEV_TIMEOUT 0x10000 /* device status word: a bounded wait gave up; low bits say where */
#define JB_DEV_LAUNCH 0x20000  /* device status word: a kernel found itself launched in another shape than its host
                                  code set (a thread-block cluster of the wrong size); low bits say which kernel */
#define JB_PRODUCT_SWIGLU 1    /* product flag: columns are gate|up blocks of 64; y = bf16(bf16(silu(g)) u) */
#define JB_PRODUCT_TMEM_A 2    /* product flag: the tensor-memory form (weights dequantised straight into tensor
                                  memory as the MMA's A operand) where it applies; the same bits, measured slower */
#define JB_PRODUCT_STATIC_MID_MAX 1048576 /* m * rank limit of jb_int4_lora_product_static (2 MiB of bf16) */

/* ABI version of this header (bumped on any signature change): 2. */
int jb_abi_version(void);
/* The message of the last failure on the calling thread ("" if none). */
const char* jb_last_error(void);
/* Reads (and with reset != 0 clears) this device's status word that kernels set when a bounded wait gives up.
 * Synchronises `stream`. Not for use inside graph capture. */
int jb_device_status(int* status, int reset, void* stream);


/* ---------------------------------------------------------------- int4 W4A16 + multi-LoRA products (S1) */

/* The reference's kernel word layout (int32 (k/8, columns); input 8i + j of column c in bits 4j..4j+3 of word
 * (i, c), stored unsigned; int4.py:215-255) -> this library's kernel layout: the same words with the nibbles of
 * inputs 0,2,4,6,1,3,5,7 in slots 0..7 (two neighbouring inputs per shift and mask). In place allowed. Load time.
 * Replaces int4.pack_kernel's output as the kernels' input (int4.py:233-255). */
int jb_int4_repack(const int32_t* words, int32_t* out, int k, int columns, void* stream);

/* Dequantise a packed group (for verification): words int32 (k/8, columns) in the kernel layout, scales and zeros
 * (nullable) bf16 (k/group, columns) -> out bf16 (columns, k), bf16(fp32(u - z) * fp32(s)) with z = 8 when zeros is
 * NULL. Replaces int4.dequantize / unpack_kernel (int4.py:203-208, :258-262). */
int jb_int4_dequant(const int32_t* words, const uint16_t* scales, const uint16_t* zeros, int k, int columns,
                    int group, uint16_t* out, void* stream);

/* LoRA first factor: mid (m, rank) bf16 = bf16(x (m, k) . A[a]^T) with fp32 accumulation in input order, A from
 * lora_a (pool_rows, rank, k) in the row a = adapters[t / row_len] of token t (an id outside [0, pool_rows) reads
 * row 0). Any row_len >= 1 when k % 128 == 0, row_len = 1 being one adapter id per token (requests of mixed lengths
 * packed back to back); a row's bits do not depend on row_len or on its neighbours. Otherwise m and row_len must be
 * multiples of 16. Replaces fast_path._lora_mid_kernel (fast_path.py:159-177) and int4_kernels._lora_mid_tile
 * (int4_kernels.py:65-82), whose tiles need row_len to be a multiple of their height (fast_path.py:225-227). */
int jb_lora_shrink(const uint16_t* x, int m, int k, const uint16_t* lora_a, int rank, int pool_rows,
                   const int32_t* adapters, int row_len, uint16_t* mid, void* stream);

/* The fused product: y (m, out) bf16 = bf16(x . W^T + mid . B[a]^T), W = dequantised int4 (kernel-layout words,
 * scales, zeros as jb_int4_dequant), the base product accumulated in fp32 by tcgen05 tensor cores from TMA-staged
 * packed weights dequantised in shared memory, then the LoRA expand (mid from jb_lora_shrink, B from lora_b (pool_rows, columns,
 * rank)) added into the same accumulator, rounded once. rank 0 (or mid NULL) leaves out the LoRA term.
 * Requires k % 64 == 0, columns % 64 == 0, out <= columns, ldy % 8 == 0 and row_len >= 1. With row_len % 128 == 0
 * the expand operands are loaded by TMA (one adapter per 128-row half); with any other row_len (down to 1: one
 * adapter id per token) they are gathered per 256-row tile from that tile's adapters, which needs pool_rows <= 256
 * and m <= 32768. Both give a row the same bits. Replaces int4_kernels.int4_product (int4_kernels.py:132-177) and
 * Lin.__call__ (fast_path.py:347-349). */
int jb_w4a16_lora(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                  const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid, const uint16_t* lora_b,
                  int rank, int pool_rows, const int32_t* adapters, int row_len, uint16_t* y, int ldy, int flags,
                  void* stream);

/* jb_w4a16_lora for passes of at most 64 tokens in at most two LoRA rows (row_len tokens each), streaming the
 * weights: one CTA per (128-column tile, K slice), every K block of its slice loaded at once (TMA) and dequantised
 * into tcgen05 MMAs with the tokens as N (m rounded up to 16); the slices of a tile are one thread-block cluster and
 * add their fp32 sums in slice order over distributed shared memory (deterministic), each storing its share of the
 * tokens. split: K slices per tile, 1, 2, 4 or 8, dividing k / 64 and leaving each slice a multiple of 4 of the
 * m-rounded-up-to-16 tokens and a slice that fits in shared memory; 0 chooses the most whose grid still fits on the
 * SMs at once. LoRA (mid given): each row's expand, its adapter's B rows by TMA. Same arguments and flags as
 * jb_w4a16_lora otherwise. Replaces int4_kernels.int4_product (int4_kernels.py:132-177) in the reference's batch-1
 * and small-batch graphs, which pick their product kernel per recorded pass (product_choice.py:1-13, 69-84). */
int jb_w4a16_lora_small(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                        const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid,
                        const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len,
                        uint16_t* y, int ldy, int flags, int split, void* stream);

/* jb_lora_shrink then jb_w4a16_lora, with the caller's scratch `mid` (at least m * rank bf16). flags: 0, or
 * JB_PRODUCT_SWIGLU for a gate/up group whose columns are interleaved in blocks of 64 (gate 64, up 64, ...): then y
 * (m, out / 2) = bf16(bf16(silu(g)) u) of the rounded products, the reference's silu_mul (fast_path.py:141-156)
 * fused into the product's epilogue. */
int jb_int4_lora_product(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                         const uint16_t* zeros, int group, int columns, int out, const uint16_t* lora_a,
                         const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len,
                         uint16_t* mid, uint16_t* y, int ldy, int flags, void* stream);

/* jb_int4_lora_product for small passes, with the caller's split scratch. Passes of at most 64 tokens in at most two
 * LoRA rows (the reference's batch-1 and two-row buckets) run jb_w4a16_lora_small with its own choice of K slices.
 * Other passes of at most 64 tokens with few tiles (at most a quarter as many 256 x 128 tiles as SMs) take the
 * persistent kernel with its K split into up to 4 slices: `partials` (partial_floats floats) holds the slices' fp32
 * sums, `counters` (counter_count int32, one per tile) must be zero before the first call and are left zero. Too
 * little scratch: fewer slices. Same result as jb_int4_lora_product up to the order of the fp32 sums (slices added
 * in slice order: deterministic). Replaces int4_kernels.int4_product (int4_kernels.py:132-177) in the reference's
 * batch-1 and small-batch graphs. */
int jb_int4_lora_product_split(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                               const uint16_t* zeros, int group, int columns, int out, const uint16_t* lora_a,
                               const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len,
                               uint16_t* mid, uint16_t* y, int ldy, int flags, float* partials,
                               int64_t partial_floats, int32_t* counters, int counter_count, void* stream);

/* jb_int4_lora_product without the `mid` argument, allocating nothing: the shrink's output goes to a scratch array
 * fixed in the library's device memory (one per device, m * rank <= JB_PRODUCT_STATIC_MID_MAX; larger calls get
 * JB_EINVAL). For callers that must not allocate device memory: a host binding the C ABI directly with no device
 * allocator of its own, or one whose device memory its own pool reserves up front. The first call on a device
 * looks up the array's address there (make it before any stream capture). Calls on one device must not overlap
 * (two streams or two host threads at once): they share the scratch and race. The scratch needs no zeroing: the
 * shrink writes all of it that the expand reads. This entry point has no counterpart in the reference, whose
 * int4_product (int4_kernels.py:132-177) keeps the LoRA intermediate in a torch-allocated Workspace buffer (ws.QP)
 * and allocates its output through torch on every call. */
int jb_int4_lora_product_static(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                                const uint16_t* zeros, int group, int columns, int out, const uint16_t* lora_a,
                                const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters,
                                int row_len, uint16_t* y, int ldy, int flags, void* stream);

/* ---------------------------------------------------------------- fused norms and activations (S4) */

/* xo = bf16(x + d) (d NULL: xo = x, may alias), h = bf16(rms(xo) * w1), w1 = 1 + weight (fp32, n). rows x n.
 * Replaces fast_path.add_rms (fast_path.py:80-100). */
int jb_add_rms(const uint16_t* x, const uint16_t* d, const float* w1, uint16_t* xo, uint16_t* h, int rows, int n,
               void* stream);
/* hidden (b, n) = bf16(rms(bf16(x[t] + d[t])) * w1) at each row's last real token t = r * row_len + last[r].
 * Replaces the final norm of batched_path.body (batched_path.py:274-275). */
int jb_rms_last(const uint16_t* x, const uint16_t* d, const int32_t* last, int b, int row_len, int n,
                const float* w1, uint16_t* hidden, void* stream);
/* x (t, dim) = table[ids] (embedding gather). Replaces embed.index_select (batched_path.py:251). */
int jb_embed(const uint16_t* table, int vocab, int dim, const int32_t* ids, int t, uint16_t* x, void* stream);
/* y (rows, inter) = bf16(bf16(silu(g)) * u), g = gu[:, :inter], u = gu[:, inter:2 inter].
 * Replaces fast_path.silu_mul (fast_path.py:141-156). */
int jb_silu_mul(const uint16_t* gu, int ldgu, int inter, uint16_t* y, int rows, void* stream);
/* y (rows, 2048) = bf16(o * bf16(sigmoid(gate))), o (rows, 8, 256), gate from pr's query/gate interleave.
 * Replaces fast_path.gate_mul (fast_path.py:123-138). */
int jb_gate_mul(const uint16_t* o, const uint16_t* pr, int ldpr, uint16_t* y, int rows, void* stream);
/* Gated DeltaNet output norm: y (rows, 2048) = bf16(bf16(w * bf16(rms(o))) * silu(z)), per head of 128,
 * z = pr[:, z_off:z_off + 2048]. Replaces fast_path.gated_norm (fast_path.py:103-120). */
int jb_gated_norm(const uint16_t* o, const uint16_t* pr, int ldpr, int z_off, const uint16_t* w, uint16_t* y,
                  int rows, void* stream);
/* Per-row readout and option softmax: probs (b, 255) fp32 from hidden (b, 1024) and the row's adapter readout
 * (pool_rows, 255, 1024) bf16: logits bf16(W h) (fp32 sums), options >= counts[r] to -1e9, / temp_pool[a], softmax.
 * Replaces batched_kernels.readout_rows (batched_kernels.py:492-559). */
int jb_readout_rows(const uint16_t* hidden, const uint16_t* readout_pool, int pool_rows, const float* temp_pool,
                    const int32_t* adapters, const int32_t* counts, int b, float* probs, void* stream);

/* ---------------------------------------------------------------- Gated DeltaNet (S2) */

/* Input side for t = b * n tokens (rows of n): causal width-4 conv over the row's 3 cached inputs (its conv page
 * tables[r][conv_entry], layer slot conv_slot) and its new ones, SiLU -> bf16, q/k L2-normalised -> bf16, v;
 * g = a_neg * softplus(a + dt_bias) fp32, beta = bf16(sigmoid(b)). pr (t, ldpr >= 8224) = [qkv | z | b | a].
 * real (nullable, the prefix pass): tokens from real[r] on get g = 0, beta = 0, and the row's last three real conv
 * inputs are written to its output conv page out_tables[r][conv_entry] (zeros first when real < 3).
 * Replaces batched_kernels.gdn_prep_rows (batched_kernels.py:89-194). */
int jb_gdn_prep_rows(const uint16_t* pr, int ldpr, int t, int n, void* pool, int64_t page_bytes,
                     const int32_t* tables, int table_stride, int conv_entry, int conv_slot, const float* conv_w,
                     const float* a_neg, const float* dt_bias, uint16_t* q, uint16_t* k, uint16_t* v, float* g,
                     uint16_t* beta, const int32_t* real, const int32_t* out_tables, int out_table_stride,
                     void* stream);
/* The gated delta rule over each row's n tokens from its state read in place from the pool (flat head
 * first_head + h at tables[r][(first_head + h) / heads_per_page], slot % heads_per_page); o (b, n, 16, 128) bf16.
 * Chunks of 64 tokens on tensor cores (bf16 operands, fp32 accumulation and state). last (nullable): outputs past
 * last[r] are written as zeros. out_tables (nullable, the prefix pass): write each row's final state into its own
 * state pages. Replaces fla's chunk_gated_delta_rule at batched_path.py:282-288, :322-324 (with the gathered initial
 * states of batched_kernels.gather_gdn_states, :264-296, read in place instead). */
int jb_gdn_scan(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const uint16_t* beta,
                uint16_t* o, int b, int n, void* pool, int64_t page_bytes, const int32_t* tables, int table_stride,
                int first_head, int heads_per_page, const int32_t* last, const int32_t* out_tables,
                int out_table_stride, void* stream);
/* The same rule with every chunk product on tcgen05 (M 128 MMAs, S and the chunk products in tensor memory, two
 * CTAs per SM), arguments and results as jb_gdn_scan (the same bf16 rounding points; fp32 sums in the tensor core's
 * order): the decision and prefix passes' scan. Replaces fla's chunk_gated_delta_rule at batched_path.py:282-288,
 * :322-324. */
int jb_gdn_scan_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const uint16_t* beta,
                   uint16_t* o, int b, int n, void* pool, int64_t page_bytes, const int32_t* tables, int table_stride,
                   int first_head, int heads_per_page, const int32_t* last, const int32_t* out_tables,
                   int out_table_stride, void* stream);
/* The same rule token by token in fp32 (one value column per thread pair): the reference's
 * batched_kernels.gdn_recurrent_slots (:200-261); last (nullable) stops after last[r], zeros past it. */
int jb_gdn_scan_recurrent(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                          const uint16_t* beta, uint16_t* o, int b, int n, void* pool, int64_t page_bytes,
                          const int32_t* tables, int table_stride, int first_head, int heads_per_page,
                          const int32_t* last, const int32_t* out_tables, int out_table_stride, void* stream);

/* A Gated DeltaNet layer's mixer in one launch: jb_gdn_prep_rows, jb_gdn_scan and jb_gated_norm fused (one CTA per
 * (row, head); q, k, v, g, beta and o stay on chip): y (t, ldy >= 2048) bf16, column block [128 h, 128 h + 128) for
 * head h, from pr (t, ldpr) = [q | k | v | z | b | a], bit-identical to the three calls in sequence. The state of
 * flat head first_head + h and the layer's conv tail (tables[r][conv_entry], slot conv_slot) are read in place;
 * last (nullable, the decision pass): outputs past last[r] are those of o = 0; real and out_tables (nullable, the
 * prefix pass): tokens from real[r] on leave the state unchanged, each row's final state and last three real conv
 * inputs go to its own pages. Replaces the Gated DeltaNet part of batched_path.body (batched_path.py:269-289:
 * gdn_prep_rows, fla's chunk_gated_delta_rule, the gated norm of fast_path.py:103-120). */
int jb_gdn_layer(const uint16_t* pr, int ldpr, int t, int n, void* pool, int64_t page_bytes, const int32_t* tables,
                 int table_stride, int first_head, int heads_per_page, int conv_entry, int conv_slot,
                 const float* conv_w, const float* a_neg, const float* dt_bias, const uint16_t* gnorm_w, uint16_t* y,
                 int ldy, const int32_t* last, const int32_t* real, const int32_t* out_tables, int out_table_stride,
                 void* stream);

/* ---------------------------------------------------------------- attention (S3) */

/* Attention input side: per token q/k per-head RMSNorm * w1 -> bf16, RoPE on the first 64 dims at position
 * pos[r] + j (inv_freq (32,) fp32; cos and sin rounded to bf16); q (t, 8, 256), kn, vn (t, 2, 256).
 * Replaces batched_kernels.attn_prep_rows (batched_kernels.py:302-364). */
int jb_attn_prep_rows(const uint16_t* pr, int ldpr, int t, int n, const float* q_w1, const float* k_w1,
                      const float* inv_freq, const int32_t* pos, uint16_t* q, uint16_t* kn, uint16_t* vn,
                      void* stream);
/* Each row's queries over its prefix (pos[r] tokens in the key/value pages tables[r][kv_entry + j / 32]) fully,
 * then its own new keys causally; GQA 8 query / 2 key-value heads of 256, softmax scale 1/16, weights rounded to
 * bf16 before the value product; out (t, 8, 256) bf16. Replaces batched_kernels.paged_attention
 * (batched_kernels.py:370-486) and the prefix pass's scaled_dot_product_attention (batched_path.py:333-336). */
int jb_paged_attention(const uint16_t* q, const void* pool, int64_t page_bytes, const int32_t* tables,
                       int table_stride, int kv_entry, int attn_layer, int attn_layers, const int32_t* pos,
                       const uint16_t* kn, const uint16_t* vn, uint16_t* out, int b, int n, void* stream);
/* Paged prefix-KV attention with the output gate, on tcgen05: y (b n, ldy >= 2048) bf16 = bf16(bf16(O) *
 * bf16(sigmoid(gate))), O the softmax(q k^T / 16) v of each query over its row's prefix keys (pool pages
 * tables[r][kv_entry + j / 32] of the pool's pool_pages pages, attention layer attn_layer) and its own new keys
 * causally, the gate the second half of each head's q_proj output in pr (t, ldpr). S and O in tensor memory, P
 * rounded to bf16 before P V. n a multiple of 32. Replaces batched_kernels.paged_attention (batched_kernels.py:
 * 370-486) followed by fast_path.gate_mul (fast_path.py:123-138). */
int jb_paged_attention_gated(const uint16_t* q, const void* pool, int64_t pool_pages, int64_t page_bytes,
                             const int32_t* tables, int table_stride, int kv_entry, int attn_layer, int attn_layers,
                             const int32_t* pos, const uint16_t* kn, const uint16_t* vn, const uint16_t* pr, int ldpr,
                             uint16_t* y, int ldy, int b, int n, void* stream);
/* jb_paged_attention_gated with each row's key walk split over several CTAs when the unsplit walk's CTAs (b x 2 x
 * n / 32) leave SMs idle (batch-1 and small passes): enough slices to cover the SMs, at most 16, as many as `scratch`
 * (scratch_floats fp32: per slice b n x 8 x 258) holds; each slice keeps its unnormalised O, running max and row
 * sum, and a combine kernel adds the slices in order (deterministic) before the same bf16 roundings and gate. The
 * same result up to the order of the fp32 sums. Replaces batched_kernels.paged_attention's split into 1/2/4/8/16
 * programs plus its combine (batched_kernels.py:370-486), chosen per graph there (batched_path.py:101-104). */
int jb_paged_attention_gated_split(const uint16_t* q, const void* pool, int64_t pool_pages, int64_t page_bytes,
                                   const int32_t* tables, int table_stride, int kv_entry, int attn_layer,
                                   int attn_layers, const int32_t* pos, const uint16_t* kn, const uint16_t* vn,
                                   const uint16_t* pr, int ldpr, uint16_t* y, int ldy, int b, int n, float* scratch,
                                   int64_t scratch_floats, void* stream);
/* The prefix pass's page scatter: each row's new keys/values (tokens below ceil(real[r] / 32) * 32) into its
 * pages out_tables[r][kv_entry + j / 32] of attention layer attn_layer. Replaces pool.kv.index_copy_
 * (batched_path.py:345-349). */
int jb_kv_scatter(const uint16_t* kn, const uint16_t* vn, int b, int n, const int32_t* real, void* pool,
                  int64_t page_bytes, const int32_t* out_tables, int table_stride, int kv_entry, int attn_layer,
                  int attn_layers, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JEFFB200_H */
