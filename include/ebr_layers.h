/* ebr_layers.h: C ABI of the fused kernels on either side of the attention in the energy network E(z; x).
 *
 * These are the callers of the attention path: the 2D-RoPE split of the qkv projection into head-major q / k / v and
 * its exact adjoint (the reference's ebr_fused::rope_split / rope_merge, models/fused_attn/rope_split.py:31-172), the
 * post-norm residual + rms_norm and the SwiGLU activation of each block (models/layers.py:37-42, :74-84,
 * models/attention.py post-norm block), and the pointwise ops of one descent microstep, v = rms_norm(z) + noise and
 * z' = sphere(v - alpha dE/dv) (models/energy.py:219-241).
 *
 * Conventions (as include/ebr_attn.h): device pointers, sizes in elements, the caller's stream as void*, nothing
 * allocated, nothing trapped. Every function returns EBR_OK (0) or an ebr_status code; ebr_attn_last_error() holds
 * the message. Arithmetic is in float32 (float64 for EBR_FLOAT64) with one rounding to the I/O type where the
 * reference's eager code rounds, so the outputs match it bit for bit up to the order of the row sums.
 */
#ifndef EBR_LAYERS_H
#define EBR_LAYERS_H

#include <stddef.h>
#include <stdint.h>

#include "ebr_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* q, k, v [B, H, N, D] (contiguous) from qkv [B, N, 3 H D] (token stride stride_n, batch stride stride_b, unit
 * channel stride): t' = t * cos + quarter_swap(t) * sin for q and k in float32, rounded once; v copied. cos / sin:
 * float32 [N, D] tables with the sign of rotate_half folded into sin (quarter_swap: (a, b, c, d) -> (b, a, d, c) over
 * the quarters of D). qscale: NULL, or float32 [H] per-head temperature already rounded to the I/O type, applied as
 * q = round(round(R q) * qscale[h]). D must be a multiple of 4.
 * Replaces: ebr_fused::rope_split / rope_split_triton.rope_split (models/fused_attn/rope_split.py:77-82, ref_split
 * :31-50). */
int ebr_rope_split(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, const void* qkv, int64_t stride_b,
                   int64_t stride_n, const float* cos_table, const float* sin_table, const float* qscale, void* q,
                   void* k, void* v, void* stream);

/* The qkv projection with the split as its epilogue (one tensor-core GEMM, the [B, N, 3 H D] projection never stored):
 * qkv = x W^T with fp32 accumulation and one rounding to the I/O type, then q, k, v exactly as ebr_rope_split makes
 * them from that qkv. x: [B N, C] rows (row stride x_stride elements, unit column stride), W: [3 H D, C] contiguous
 * (the nn.Linear weight in the I/O type). bfloat16 / float16 only; D = 64 or 128, H D a multiple of 256, C a multiple
 * of 64, x_stride a multiple of 8 and every pointer 16-byte aligned, else EBR_ERR_SHAPE / EBR_ERR_STRIDE (the caller
 * then runs its GEMM and ebr_rope_split). Replaces: F.linear + rope_split in EnergyAttention
 * (models/attention.py:233-242, models/fused_attn/rope_split.py:77-82). */
int ebr_qkv_rope_split(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, int64_t C, const void* x,
                       int64_t x_stride, const void* w, const float* cos_table, const float* sin_table,
                       const float* qscale, void* q, void* k, void* v, void* stream);

/* The input gradient of the qkv projection with the RoPE merge folded in: dx = rope_merge(dq, dk, dv) W, the
 * [B, N, 3 H D] merged gradient (ebr_rope_merge's output, rounded to the I/O type) never stored. dq / dk / dv:
 * [B, H, N, D] operands (16-byte aligned data and strides, unit head-dim stride); w: the [3 H D, C] projection weight,
 * contiguous; cos / sin: float32 [N, D] tables; qscale: NULL or float32 [H] (applied to dq first, as ebr_rope_merge
 * does); addend: NULL or [B, N, C] contiguous, added to the rounded product and rounded again (a residual gradient
 * joined in, as a separate add of the two would); dx: [B, N, C] contiguous. bfloat16 / float16 only, D = 64 and
 * C = 512, else EBR_ERR_SHAPE / EBR_ERR_STRIDE
 * (the caller then runs ebr_rope_merge and its GEMM). Replaces: rope_merge + the linear layer's input gradient in the
 * backward of EnergyAttention (models/fused_attn/rope_split.py:84-96). */
int ebr_qkv_rope_merge_dx(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, int64_t C, const ebr_operand* dq,
                          const ebr_operand* dk, const ebr_operand* dv, const void* w, const float* cos_table,
                          const float* sin_table, const float* qscale, const void* addend, void* dx,
                          void* stream);

/* The attention's output projection from the head-major attention output: y[b, n, :] = sum_h O[b, h, n, :] W_h^T with
 * W_h = W[:, h D : (h + 1) D], fp32 accumulation and one rounding to the I/O type (the [B, N, H D] transpose of O is
 * never stored). o: [B, H, N, D] operand (16-byte aligned data and strides, unit head-dim stride); w: [C_out, H D]
 * contiguous; y: [B, N, C_out] contiguous. bfloat16 / float16 only, D = 64 or 128, C_out a multiple of 256, else
 * EBR_ERR_SHAPE / EBR_ERR_STRIDE (the caller then transposes O and runs its GEMM). Replaces:
 * self.o(y.transpose(1, 2).reshape(b, n, h d)) in EnergyAttention (models/attention.py:241-242). */
int ebr_o_proj(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, int64_t C_out, const ebr_operand* o,
               const void* w, void* y, void* stream);

/* The adjoint: dqkv [B, N, 3 H D] (contiguous) from dq, dk, dv (strided [B, H, N, D] operands): dq is first scaled
 * by qscale (if not NULL) and rounded, then g' = g * cos + quarter_swap(g * sin) for dq and dk, rounded once; dv
 * copied. Replaces: ebr_fused::rope_merge (models/fused_attn/rope_split.py:91-96, ref_merge :53-67). */
int ebr_rope_merge(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, const ebr_operand* dq,
                   const ebr_operand* dk, const ebr_operand* dv, const float* cos_table, const float* sin_table,
                   const float* qscale, void* dqkv, void* stream);

/* Residual + rms_norm over rows of C contiguous elements:
 *   s = round(x + a)            (a may be NULL: s = x; sum_out may be NULL, else s is written there)
 *   y = round(s * rsqrt(mean(s^2) + eps)),  rstd_out[row] = rsqrt(mean(s^2) + eps) (float32; may be NULL)
 *   if post != NULL: y = round(y + round(post * post_scale))   (the descent point v = rms_norm(z) + noise * sigma)
 * Replaces: rms_norm(x + sublayer(x)) of the post-norm block and the descent state normalisation
 * (models/layers.py:37-42; models/energy.py:226-232, :322-341). */
int ebr_add_rms_norm(int dtype, int64_t rows, int64_t C, double eps, const void* x, const void* a, void* sum_out,
                     void* y, float* rstd_out, const void* post, double post_scale, void* stream);

/* Backward of ebr_add_rms_norm (without post): gs = round(rstd * (gy - xh * mean(gy * xh))), xh = s * rstd; gs is
 * the gradient of both x and a. */
int ebr_rms_norm_bwd(int dtype, int64_t rows, int64_t C, const void* s, const float* rstd, const void* gy, void* gs,
                     void* stream);

/* Double backward of ebr_rms_norm_bwd, for second-order training: given the upstream gradient u of gs, with n = C,
 * r = rstd and the row sums U_g = sum u gy, U_s = sum u s, G = sum gy s: dgy = r u - (r^3 / n) s U_s and
 * ds = (r^3 / n) (-s U_g + 3 r^2 s G U_s / n - G u - gy U_s) (ds is the gradient of both x and a). */
int ebr_rms_norm_bwd2(int dtype, int64_t rows, int64_t C, const void* s, const float* rstd, const void* gy,
                      const void* u, void* ds, void* dgy, void* stream);

/* SwiGLU activation over rows of 2 I: out[r, j] = round(round(silu(h[r, j])) * h[r, I + j]), out [rows, I].
 * Replaces: F.silu(gate) * up after gate_up_proj(x).chunk(2) (models/layers.py:82-84). */
int ebr_swiglu_fwd(int dtype, int64_t rows, int64_t I, const void* h, void* out, void* stream);

/* The MLP's gate / up projection with the activation as its epilogue (one tensor-core GEMM): h = x W^T [rows, 2 I]
 * (fp32 accumulation, one rounding to the I/O type; gate columns [0, I), up columns [I, 2 I)) and act [rows, I] exactly
 * as ebr_swiglu_fwd makes it from that h. x: [rows, C] (row stride x_stride elements), W: [2 I, C] contiguous.
 * bfloat16 / float16 only; C a multiple of 64, I a multiple of 128, x_stride a multiple of 8, 16-byte aligned
 * pointers, else EBR_ERR_SHAPE / EBR_ERR_STRIDE. Replaces: gate_up_proj(x) and F.silu(gate) * up
 * (models/layers.py:80-84). */
int ebr_gate_up_swiglu(int dtype, int64_t rows, int64_t C, int64_t I, const void* x, int64_t x_stride, const void* w,
                       void* h, void* act, void* stream);

/* Its backward: gh [rows, 2 I] = (silu'(gate) * round(gout * up), round(gout * round(silu(gate)))). */
int ebr_swiglu_bwd(int dtype, int64_t rows, int64_t I, const void* h, const void* gout, void* gh, void* stream);

/* Double backward of ebr_swiglu_bwd, for second-order training (a graph built through the backward): given the
 * upstream gradient u [rows, 2 I] of gh, dh [rows, 2 I] = (u_g da s2 + u_u gout s1, u_g gout s1) and dgout [rows, I]
 * = u_g up s1 + u_u act, with s1 = silu'(gate), s2 = silu''(gate), da = round(gout up), act = round(silu(gate)). */
int ebr_swiglu_bwd2(int dtype, int64_t rows, int64_t I, const void* h, const void* gout, const void* u, void* dh,
                    void* dgout, void* stream);

/* One descent step and projection, z' = sphere(v - alpha * g) over rows of `row_elems` elements (a whole board:
 * N * C): u = round(v - round(alpha * g)), z' = round(u / max(sqrt(mean(u^2)), eps)). `partial` is float32 scratch
 * of ebr_descent_step_scratch_floats(rows, row_elems) elements (the caller allocates it). Replaces: _step_and_project
 * and sphere (models/energy.py:219-241). */
int ebr_descent_step(int dtype, int64_t rows, int64_t row_elems, double alpha, double eps, const void* v,
                     const void* g, void* z_next, float* partial, size_t partial_floats, void* stream);
size_t ebr_descent_step_scratch_floats(int64_t rows, int64_t row_elems);

#ifdef __cplusplus
}
#endif

#endif /* EBR_LAYERS_H */
