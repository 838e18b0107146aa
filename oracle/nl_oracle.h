/* nl_oracle.h -- CPU restatement of the nelisp-gpu hot-path kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker and the
 * timed CPU baseline; it is never linked into libnelisp_cuda and no product
 * code path calls it.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load it.
 *
 * Every function restates one DSL kernel of the reference
 * (lisp/nelisp-gpu-kernels.el in zawatton/nelisp-gpu) with the same f32
 * operation order, compiled with -ffp-contract=off so no multiply-add is
 * fused that the reference's SPIR-V kept separate.  The reference runs one
 * GPU invocation per output element; here that becomes an OpenMP
 * `parallel for` over the same decomposition.  Buffers are the reference's:
 * raw little-endian 32-bit words, f32 unless the kernel bit-casts them.
 */
#ifndef NL_ORACLE_H
#define NL_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

int  nlo_threads(void);                 /* OpenMP threads the oracle uses */
void nlo_set_threads(int n);

/* ternary-rows, lisp/nelisp-gpu-kernels.el:713-746 */
void nlo_ternary_rows(const float *X, const uint32_t *WP, const float *BIAS,
                      const float *BETA, float *Y, uint32_t seq, uint32_t out,
                      uint32_t cols, uint32_t nblk, uint32_t wng);
/* ternary-rows-t, lisp/nelisp-gpu-kernels.el:750-772 */
void nlo_ternary_rows_t(const uint32_t *WP, const float *BETA, const float *G,
                        float *X, uint32_t out, uint32_t cols, uint32_t nblk,
                        uint32_t wng, uint32_t seq);
/* y[s,o] = s[o] * sum_i t(o,i) x[s,i]: ternary-rows with one scale per row
 * replicated into every 128-column block and a zero bias. */
void nlo_ternary_gemv_rows(const float *X, const uint32_t *WP, const float *S,
                           float *Y, uint32_t seq, uint32_t out, uint32_t cols);
/* bitlinear-packed (per_row=0, :998-1016) / bitlinear-packed-v (per_row=1,
 * :1022-1040) */
void nlo_bitlinear_packed(const float *X, const float *WPK, const float *BIAS,
                          const float *BETA, float *Y, uint32_t seq,
                          uint32_t in, uint32_t out, uint32_t pk,
                          uint32_t fcount, int per_row);
/* pack-act-rows, :898-932 */
void nlo_pack_act_rows(const float *X, uint32_t *XQ, float *GAMMA,
                       uint32_t seq, uint32_t cols, uint32_t ng);
/* bitlinear-dp4a-1f (per_row=0, :623-634) / bitlinear-dp4a-rows
 * (per_row=1, :642-653) */
void nlo_dp4a_rows(const uint32_t *AP, const uint32_t *WP, const float *BIAS,
                   const float *BETA, const float *GAMMA, float *Y,
                   uint32_t seq, uint32_t out, uint32_t ng, int per_row);
/* matmul :17-27, linear :71-81, matmul-tiled :82-107, matmul-reg :129 */
void nlo_matmul(const float *A, const float *B, float *C, uint32_t M,
                uint32_t K, uint32_t N);
void nlo_matmul_tiled(const float *A, const float *B, float *C, uint32_t M,
                      uint32_t K, uint32_t N);
void nlo_matmul_reg(const float *A, const float *B, float *C, uint32_t M,
                    uint32_t K, uint32_t N);
void nlo_linear(const float *X, const float *W, const float *B, float *C,
                uint32_t M, uint32_t IN, uint32_t OUT);
/* softmax :28-42 */
void nlo_softmax(const float *A, float *C, uint32_t M, uint32_t N);
/* silu-mul :187-193, add2 :816-821, scale :141 */
void nlo_silu_mul(const float *A, const float *B, float *C, uint32_t n);
void nlo_add2(const float *A, const float *B, float *C, uint32_t n);
void nlo_scale(const float *A, const float *S, float *C, uint32_t n);
/* rmsnorm-istd :1250-1256 (eps 1e-6, as the reference hard-codes),
 * rmsnorm-fwd :1259-1265 */
void nlo_rmsnorm_istd(const float *X, float *S, uint32_t M, uint32_t N);
void nlo_rmsnorm_fwd(const float *X, const float *S, const float *G, float *C,
                     uint32_t M, uint32_t N);
/* rope-half :857-882; rbase and sgn are f32 bit patterns */
void nlo_rope_half(const float *X, float *Y, uint32_t seq, uint32_t nheads,
                   uint32_t hd, uint32_t rbase_bits, uint32_t sgn_bits);
/* decode-rope-b :342-355 (decode-rope :294 is B=1) */
void nlo_decode_rope_b(const float *X, const float *CO, const float *SI,
                       const float *SG, const float *POS, float *C,
                       uint32_t B, uint32_t cols, uint32_t heads);
/* cache-append-b :358-365 (cache-append :308 is B=1, maxseq unused) */
void nlo_cache_append_b(const float *SRC, const float *POS, float *CACHE,
                        uint32_t B, uint32_t kvdim, uint32_t maxseq);
/* decode-attn-b :368-390 (decode-attn :317-338 is B=1) */
void nlo_attn_causal_gqa(const float *Q, const float *K, const float *V, float *CTX,
                         uint32_t seq, uint32_t heads, uint32_t kvheads, uint32_t hd);
void nlo_cache_append_ring(const float *SRC, const float *POS, float *CACHE, uint32_t kvdim,
                           uint32_t nsink, uint32_t win);
void nlo_qkv_append(const float *QKV, float *CK, float *CV, uint32_t dim, uint32_t kvdim,
                    uint32_t wbase);
void nlo_cache_append_paged(const float *SRC, const float *POS, const float *LENS,
                            const float *TABLE, float *POOL, uint32_t B, uint32_t kvdim,
                            uint32_t bs, uint32_t mbps);
void nlo_block_copy(float *POOL, uint32_t bs, uint32_t kvdim, uint32_t src, uint32_t dst);
void nlo_decode_rope_b_v(const float *X, const float *CO, const float *SI, const float *SG,
                         const float *LENS, float *C, uint32_t B, uint32_t cols, uint32_t heads);
void nlo_decode_attn_stream(const float *Q, const float *CK, const float *CV, const float *POS,
                            const float *CO, const float *SI, float *C, uint32_t dim,
                            uint32_t heads, uint32_t kvheads, uint32_t nsink, uint32_t win);
void nlo_attn_stream_entries(const float *Q, const float *CK, const float *CV, const float *ENT,
                             const float *CO, const float *SI, float *C, uint32_t dim,
                             uint32_t heads, uint32_t kvheads, uint32_t ne, uint32_t qcrel);
void nlo_decode_attn_paged(const float *Q, const float *CK, const float *CV, const float *POS,
                           const float *LENS, const float *TABLE, float *C, uint32_t B,
                           uint32_t dim, uint32_t heads, uint32_t kvheads, uint32_t bs,
                           uint32_t mbps);
void nlo_decode_attn_b(const float *Q, const float *CK, const float *CV,
                       const float *POS, float *C, uint32_t B, uint32_t dim,
                       uint32_t heads, uint32_t kvheads, uint32_t maxseq);
/* embed-gather :1385-1392 */
void nlo_embed_gather(const float *TOK, const float *WTE, float *C,
                      uint32_t seq, uint32_t dim);

/* nl_oracle_misc.c: matmul-at :177-186, causal-mask :148-155, attn-scores
 * :208-221, attn-context :224-235, dp4a-dot :592-602, bitlinear-dp4a :606-620,
 * dp4a-rows-t :792-810, rmsnorm-heads :828-845, rope-apply :1290-1303, silu
 * :1306-1312, scale-rows :1365-1372 */
void nlo_matmul_at(const float *A, const float *B, float *C, uint32_t M, uint32_t K,
                   uint32_t N);
void nlo_causal_mask(float *S, uint32_t n);
void nlo_attn_scores(const float *Q, const float *K, float *S, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads);
void nlo_attn_context(const float *P, const float *V, float *C, uint32_t seq, uint32_t dim,
                      uint32_t heads, uint32_t kvheads);
void nlo_dp4a_dot(const float *ALO, const float *AHI, const float *BLO, const float *BHI,
                  float *OUT, uint32_t n);
void nlo_bitlinear_dp4a(const float *ALO, const float *AHI, const float *WLO, const float *WHI,
                        const float *BIAS, const float *BETA, const float *GAMMA, float *Y,
                        uint32_t seq, uint32_t out, uint32_t ng);
void nlo_dp4a_rows_t(const float *WP, const float *BETA, const float *G, float *X, uint32_t out,
                     uint32_t cols, uint32_t ng, uint32_t seq);
void nlo_rmsnorm_heads(const float *X, const float *G, float *Y, uint32_t seq, uint32_t nheads,
                       uint32_t hd);
void nlo_rope_apply(const float *X, const float *CO, const float *SI, const float *SG, float *C,
                    uint32_t seq, uint32_t dim, uint32_t heads);
void nlo_silu(const float *X, float *C, uint32_t n);
void nlo_scale_rows(const float *Y, const float *S, float *C, uint32_t M, uint32_t N);
/* nl_oracle_misc.c: sumsq-acc :496-503, clip-scale :505-512, absmean-acc
 * :516-526, quant-act :529-548, quant-w :550-561, and the repacking of
 * nl_upload_file_ternary */
void nlo_sumsq_acc(const float *G, float *ACC, uint32_t n);
void nlo_absmean_acc(const float *G, float *ACC, uint32_t n);
void nlo_clip_scale(const float *GSQ, const float *CFG, float *SCALE);
void nlo_quant_act(const float *X, float *XQ, uint32_t seq, uint32_t cols);
void nlo_quant_w(const float *W, const float *S, float *WQ, uint32_t n);
void nlo_quant_w_pack(const float *W, uint32_t rows, uint32_t cols, int per_row, uint32_t *WP,
                      float *S);
/* nl_oracle_misc.c: the training-side operators */
void nlo_transpose(const float *A, float *C, uint32_t R, uint32_t Co);
void nlo_slice_cols(const float *A, float *C, uint32_t seq, uint32_t dim, uint32_t hd, uint32_t c0);
void nlo_set_cols(float *D, const float *S, uint32_t seq, uint32_t dim, uint32_t hd, uint32_t c0);
void nlo_silu_mul_bwd(const float *G, const float *A, const float *B, float *DA, float *DB, uint32_t n);
void nlo_silu_bwd(const float *G, const float *X, float *D, uint32_t n);
void nlo_gelu_bwd(const float *G, const float *H, float *D, uint32_t n);
void nlo_sub_scale(const float *A, const float *B, const float *S, float *C, uint32_t n);
void nlo_sgd(float *W, const float *G, const float *L, const float *S, uint32_t n);
void nlo_adam(float *W, const float *G, float *M, float *V, const float *H, const float *S,
              uint32_t n);
void nlo_colsum(const float *G, float *D, uint32_t M, uint32_t N);
void nlo_rmsnorm_dgamma(const float *DY, const float *X, const float *S, float *DG, uint32_t M,
                        uint32_t N);
void nlo_rmsnorm_dx(const float *DY, const float *X, const float *S, const float *G, float *DX,
                    uint32_t M, uint32_t N);
void nlo_softmax_bwd(const float *P, const float *G, float *DS, uint32_t M, uint32_t N);
void nlo_rowdot(const float *G, const float *Y, float *D, uint32_t M, uint32_t N);
void nlo_ce_grad(const float *LG, const float *T, float *G, uint32_t M, uint32_t V, int idx);
void nlo_topk_mask(const float *LG, float *MK, uint32_t M, uint32_t E, uint32_t K);
void nlo_embed_bwd(const float *TOK, const float *GX, float *DW, uint32_t seq, uint32_t dim,
                   uint32_t vocab);
void nlo_gather_spike(const float *TABLE, const float *POOL, float *OUT, uint32_t n, uint32_t bs,
                      uint64_t pool_words);
void nlo_scatter_spike(const float *TABLE, const float *SRC, float *POOL, uint32_t n, uint32_t bs,
                       uint64_t pool_words);
void nlo_gdn_step(float *S, const float *Q, const float *K, const float *V, const float *G,
                  const float *B, float *OUT, uint32_t nv, uint32_t dk, uint32_t dv, uint32_t t);
void nlo_attn_sc_dq(const float *DS, const float *K, float *DQ, uint32_t seq, uint32_t dim,
                    uint32_t heads, uint32_t kvheads);
void nlo_attn_sc_dk(const float *DS, const float *Q, float *DK, uint32_t seq, uint32_t dim,
                    uint32_t heads, uint32_t kvheads);
void nlo_attn_ctx_dp(const float *DC, const float *V, float *DP, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads);
void nlo_attn_ctx_dv(const float *DC, const float *P, float *DV, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads);
void nlo_tree_attn(const float *Q, const float *CK, const float *CV, const float *NK,
                   const float *NV, const float *PAR, const float *LEN, float *C, uint32_t M,
                   uint32_t dim, uint32_t heads, uint32_t kvheads, uint32_t maxdepth);

/* Double-precision references used by the reference's own self-checks. */
double nlo_matmul_sample_ref(uint32_t r, uint32_t c, uint32_t K, uint32_t N);
void   nlo_softmax_ref_f64(const double *A, double *C, uint32_t M, uint32_t N);

#ifdef __cplusplus
}
#endif
#endif
