// C interface of the sm_100a kernels.  Every function takes raw device pointers and a stream, performs no
// allocation, and returns 0 on success or a negative code when the launch could not be made.  Kernels that
// can wait on another agent additionally take a device `status` word that is 0 unless a bounded wait ran out.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

enum ObEpilogue : int {
  EPI_BF16 = 0,       // C(bf16)  = acc
  EPI_F32_ACCUM = 1,  // C(fp32) += acc
  EPI_BF16_ADD = 2,   // C(bf16)  = acc + R(bf16), R has the pitch of C and may alias it
  EPI_F32_STORE = 3,  // C(fp32)  = acc
};

#ifdef __cplusplus
extern "C" {
#endif

// ---- gemm.cu
int ob_gemm_bf16(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb, int ldc,
                 int a_mn_major, int b_mn_major, int epi, const int* b_ready, int rows_per_flag, int ready_value,
                 int* status, int num_sms, cudaStream_t stream);

int ob_gemm_bf16_comm(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb, int ldc,
                      int a_mn_major, int b_mn_major, int epi, int* status, int num_sms, const void* task, int comm_ctas,
                      cudaStream_t stream);

// ---- gemm_smallm.cu: y[M, N] = x[M, K] · w[N, K]ᵀ for 1 <= M <= 256 (weights streamed as the 128-row operand)
int ob_gemm_smallm_splits(int N, int K, int num_sms);
int ob_gemm_smallm(const void* x, const void* w, void* y, float* partial, int M, int N, int K, int ldx, int ldw, int splits,
                   int* status, cudaStream_t stream);

// ---- attention.cu
int ob_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int T, int H, int Hkv, int q_sb,
                     int q_st, int q_sh, int k_sb, int k_st, int k_sh, int v_sb, int v_st, int v_sh, int o_sb, int o_st,
                     int o_sh, float scale, int causal, int* status, const int* doc_start, cudaStream_t stream);
int ob_attention_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse, void* dq,
                     void* dk, void* dv, float* delta, float* dq_acc, int B, int T, int H, int Hkv, int do_sb, int do_st,
                     int do_sh, int q_sb, int q_st, int q_sh, int k_sb, int k_st, int k_sh, int v_sb, int v_st, int v_sh,
                     int o_sb, int o_st, int o_sh, int dq_sb, int dq_st, int dq_sh, int dk_sb, int dk_st, int dk_sh,
                     int dv_sb, int dv_st, int dv_sh, float scale, int causal, int* status, const int* doc_start,
                     cudaStream_t stream);
// doc_start (optional, causal only): int32 [B, T], position of the first token of the document each token belongs to.
void ob_set_gemm_pair_mode(int on);  // 1: two-CTA (cta_group::2) GEMM kernel where applicable
int ob_get_gemm_pair_mode(void);
void ob_set_gemm_tma_store(int on);   // 1 (default): the two-CTA GEMM writes its output tiles through shared memory and TMA stores

// ---- comm.cu (peer-memory collectives; `task` points at an ob::CommTask, see comm.cuh)
int ob_comm_task_size(void);
int ob_comm_launch(const void* task, int nctas, cudaStream_t stream);
int ob_signal(int* flag, int value, cudaStream_t stream);
int ob_wait_flags(const void* const* flags, int n, int value, int* status, long long wait_cycles, cudaStream_t stream);
int ob_scalar_slots_bytes(void);
int ob_allreduce_scalar(const float* value, void* const* peers, void* mine, float* out, int rank, int world, int epoch,
                        int* status, long long wait_cycles, cudaStream_t stream);

// ---- norm.cu
int ob_norm_rows_per_launch(int M);
int ob_norm_fwd(const void* x, const void* res, const void* w, const void* b, void* out, float* rstd, float* mean, int M,
                int D, int ldx, float eps, int is_rms, cudaStream_t stream);
int ob_norm_bwd(const void* dy, const void* x, const void* w, const float* rstd, const float* mean, const void* dres,
                void* dx, float* dw_part, float* db_part, int M, int D, int ldx, int lddx, int is_rms,
                cudaStream_t stream);
int ob_reduce_rows_f32(const float* part, int nparts, int D, float* out, int accumulate, cudaStream_t stream);

// ---- rope.cu
int ob_qk_rows_per_launch(int M);
int ob_qk_norm_rope_fwd(const void* qkv, void* qk_out, const void* wq, const void* wk, const float* cos_t,
                        const float* sin_t, float* rstd_q, float* rstd_k, int M, int T, int pos_offset, int Wq, int Wk,
                        int hd, int ldq, int ldo, float eps, float clip, int do_norm, int do_rope, cudaStream_t stream);
int ob_qk_norm_rope_bwd(const void* qkv, void* dqkv, const void* wq, const void* wk, const float* cos_t,
                        const float* sin_t, const float* rstd_q, const float* rstd_k, float* dwq_part, float* dwk_part,
                        int M, int T, int pos_offset, int Wq, int Wk, int hd, int ldq, float clip, int do_norm,
                        int do_rope, cudaStream_t stream);

// ---- pointwise.cu
int ob_swiglu_fwd(const void* h, void* out, int M, int H, cudaStream_t stream);
int ob_swiglu_bwd(const void* dout, const void* h, void* dh, int M, int H, cudaStream_t stream);
int ob_embedding_fwd(const long long* ids, const void* table, void* out, int M, int D, int V, cudaStream_t stream);
int ob_embedding_bwd(const long long* ids, const void* dout, float* grad, int M, int D, int V, cudaStream_t stream);
int ob_accum_bf16_to_f32(const void* src, float* acc, long long n, cudaStream_t stream);
int ob_cast_f32_to_bf16(const float* src, void* dst, long long n, cudaStream_t stream);

// ---- loss_optim.cu
int ob_cross_entropy(void* logits, const long long* labels, float* ce_out, float* z_out, int R, int V, int ld,
                     long long ignore_index, float z_mult, float grad_scale, int write_grad, cudaStream_t stream);
int ob_adamw(float* p, const float* g, float* m, float* v, void* p_lowp, long long n, const long long* seg_end,
             const float* seg_wd, const float* seg_lr, int nseg, float beta1, float beta2, float eps, int step,
             const float* gscale, cudaStream_t stream);
int ob_lionw(float* p, const float* g, float* m, void* p_lowp, long long n, const long long* seg_end,
             const float* seg_wd, const float* seg_lr, int nseg, float beta1, float beta2, const float* gscale,
             cudaStream_t stream);
int ob_sumsq_num_partials(long long n);
int ob_sumsq_f32(const float* g, long long n, float* partials, float* out, int accumulate, cudaStream_t stream);
int ob_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm_out, cudaStream_t stream);

// 4-bit weight / bf16 activation inference (w4a16.cu).  qweight [N, K/8] int32, scales [N, K/G] bf16, zeros [N, K/G] uint8.
int ob_w4a16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, int M, int N, int K, int group,
                  cudaStream_t stream);  // 1 <= M <= 8
int ob_w4a16_dequant(const void* qweight, const void* scales, const void* zeros, void* out, int N, int K, int group, cudaStream_t stream);
// Fused dequantise -> tcgen05 GEMM for 1..256 activation rows (w4a16_mma.cu); `status` is the library's status word.
int ob_w4a16_gemm_small_supported(int M, int N, int K, int group);
int ob_w4a16_gemm_small_splits(int N, int K);
// Single-token decode against preallocated key/value windows (decode.cu).
int ob_decode_qkv(const void* qkv, const void* wq, const void* wk, const float* cos_t, const float* sin_t, const long long* rope_pos,
                  const long long* write_col, void* q_out, void* k_cache, void* v_cache, int R, int Wq, int Wk, int hd, int window,
                  int table_len, float eps, float clip, int qk_norm, int rope, cudaStream_t stream);
int ob_decode_attention(const void* q, const void* k_cache, const void* v_cache, const void* bias, void* out, int R, int H, int Hkv, int hd,
                        int window, int length, float scale, cudaStream_t stream);
int ob_w4a16_gemm_small(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, float* partial, int M, int N,
                        int K, int group, int splits, int* status, cudaStream_t stream);
int ob_gather_columns_bf16(const void* x, const int* perm, void* out, int M, int K, cudaStream_t stream);
// 2-, 3-, 4- and 8-bit weights as a little-endian bit stream per row (wna16.cu): qweight [N, K*bits/32] int32.
int ob_wna16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, int M, int N, int K, int group,
                  int bits, cudaStream_t stream);  // 1 <= M <= 8
int ob_wna16_dequant(const void* qweight, const void* scales, const void* zeros, void* out, int N, int K, int group, int bits,
                     cudaStream_t stream);

#ifdef __cplusplus
}
#endif
