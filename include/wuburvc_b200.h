/* wuburvc_b200.h — C ABI of the B200 (sm_100a) generator training library.
 *
 * Plain C types only: pointers, sizes, ints and floats.  Two groups of entry points:
 *
 *  1. Convolution primitives on device buffers (channels-last [B][T][C] bf16 activations).
 *     They replace the per-op kernels of the reference's CUDA trainer:
 *       k_conv1d        src/wubu_rvc_cuda.cu:36-53      -> wubu_b200_conv1d
 *       tk_conv1d_bwd   src/wubu_train_cuda.cu:67-105   -> wubu_b200_conv1d (flipped weights, dgrad)
 *                                                          + wubu_b200_conv1d_wgrad
 *       k_convt1d       src/wubu_rvc_cuda.cu:55-78      -> wubu_b200_convT
 *       tk_convt1d_bwd  src/wubu_train_cuda.cu:107-135  -> wubu_b200_convT_dgrad + wubu_b200_convT_wgrad
 *
 *  2. The generator training step (wubu_b200_gen_*): forward, backward and the fused AdamW
 *     update over one flat parameter buffer, replacing wubu_train_forward_cuda /
 *     wubu_train_backward_cuda / wubu_train_step_cuda (src/wubu_train.h:92-104).
 *
 * Return codes: 0 = OK, negative = error (see WUBU_B200_ERR_*).  Nothing here allocates on
 * behalf of the caller except where stated; every call is synchronous unless it says so.
 */
#ifndef WUBURVC_B200_H
#define WUBURVC_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define WUBU_B200_OK 0
#define WUBU_B200_ERR_ARG (-1)
#define WUBU_B200_ERR_CUDA (-2)
#define WUBU_B200_ERR_SHAPE (-3)
#define WUBU_B200_ERR_TIMEOUT (-4) /* a kernel's bounded wait expired; the context stays usable */
#define WUBU_B200_ERR_COMM (-5)
#define WUBU_B200_ERR_NOMEM (-6)

/* ---------------------------------------------------------------------------------------
 * 1. convolution primitives (device pointers, `stream` = cudaStream_t or NULL)
 * ------------------------------------------------------------------------------------- */

/* Conv1d, stride 1: out[b,t,o] = bias[o] + sum_{tap,i} x[b, t-pad+dil*tap, i] * w[tap,o,i]
 *   x_hi/x_lo [B][T][C_in] bf16, w_hi/w_lo [k][C_out][C_in] bf16, out [B][T_out][C_out] f32,
 *   T_out = T + 2*pad - dil*(k-1).  split=1: bf16x3 (hi*hi + lo*hi + hi*lo), else hi only.
 *   Replaces k_conv1d (src/wubu_rvc_cuda.cu:36-53) and conv1d_fwd (src/wubu_train.c:461-486). */
int wubu_b200_conv1d(const void* x_hi, const void* x_lo, const void* w_hi, const void* w_lo,
                     const float* bias, float* out, int B, int C_in, int T, int C_out, int k, int dil,
                     int pad, int split, void* stream);

/* Conv1d weight gradient dw[o][i][tap] = sum_{b,t} dy[b,t,o] * x[b, t-pad+dil*tap, i]
 *   dy [B][T_out][C_out] bf16, x [B][T][C_in] bf16, dw f32.
 *   Replaces the dw part of tk_conv1d_bwd (src/wubu_train_cuda.cu:67-105), conv1d_bwd
 *   (src/wubu_train.c:490-527). */
int wubu_b200_conv1d_wgrad(const void* dy, const void* x, float* dw, int B, int C_in, int T, int C_out,
                           int k, int dil, int pad, void* stream);

/* ConvTranspose1d (polyphase): out[b, i*s-pad+tap, o] += x[b,i,c] * W[c][o][tap]
 *   x [B][T_in][C_in] bf16; wp [k][C_out][C_in] bf16 = W taps in phase order
 *   (phase r = 0..s-1, taps r, r+s, r+2s, ...), transposed; out [B][T_in*s][C_out] f32.
 *   Requires k - 2*pad == s.  Replaces k_convt1d (src/wubu_rvc_cuda.cu:55-78), convt1d_fwd
 *   (src/wubu_train.c:533-562). */
int wubu_b200_convT(const void* x_hi, const void* x_lo, const void* wp_hi, const void* wp_lo,
                    const float* bias, float* out, int B, int C_in, int T_in, int C_out, int k,
                    int stride, int pad, int split, void* stream);

/* ConvTranspose1d input gradient dx[b,i,c] = sum_{tap,o} dy[b, i*s-pad+tap, o] * W[c][o][tap]
 *   dy [B][T_in*s][C_out] bf16, wd [k][C_in][C_out] bf16, dx [B][T_in][C_in] f32.
 *   Replaces the din part of tk_convt1d_bwd (src/wubu_train_cuda.cu:107-135). */
int wubu_b200_convT_dgrad(const void* dy, const void* wd, float* dx, int B, int C_in, int T_in,
                          int C_out, int k, int stride, int pad, void* stream);

/* ConvTranspose1d weight gradient dw[c][o][tap] = sum_{b,i} x[b,i,c] * dy[b, i*s-pad+tap, o]
 *   Replaces the dw part of tk_convt1d_bwd (src/wubu_train_cuda.cu:107-135). */
int wubu_b200_convT_wgrad(const void* x, const void* dy, float* dw, int B, int C_in, int T_in,
                          int C_out, int k, int stride, int pad, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WUBURVC_B200_H */
