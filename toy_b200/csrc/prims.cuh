// The tnn_* primitive op graph (graph.cu): node types, constructors with ggml
// shape semantics, realize / compute / autograd, tensor I/O.
#pragma once
#include "session.cuh"

namespace tb2 {

enum PrimOp : int {
  kOpNone = 0, kOpAdd, kOpSub, kOpMul, kOpScale, kOpSilu, kOpSiluBack, kOpSwiglu, kOpMulMat, kOpOutProd, kOpMulMatAT,
  kOpRmsNorm, kOpRmsNormBack, kOpRope, kOpRopeBack, kOpSoftMax, kOpSoftMaxBack, kOpDiagMaskInf, kOpDiagMaskZero,
  kOpTranspose, kOpCont, kOpReshape, kOpView, kOpConcat, kOpSlice, kOpGetRows, kOpGetRowsBack, kOpCrossEntropy,
  kOpCrossEntropyBack, kOpSum, kOpSumRows, kOpRepeat, kOpRepeatBack, kOpOptAdamw, kOpAccView, kOpDequant, kOpOptSgd,
  kOpMulMatId, kOpAddId, kOpArgsort, kOpTopK, kOpDetach, kOpCpy, kOpSetRows, kOpCount
};
const char* prim_op_name(int op);

// tensors (type: 0 f32, 8 q8_0, 26 i32); persistent tensors get storage now
Tensor* prim_new(Session* s, int type, int ne0, int ne1, int ne2, int ne3, int op, bool persistent);
int prim_alloc(Session* s, Tensor* t);
int prim_zero(Session* s, Tensor* t);
int prim_upload_f64(Session* s, Tensor* t, const double* data, size_t n);
int prim_upload_i64(Session* s, Tensor* t, const long* data, size_t n);
int prim_upload_q8_0(Session* s, Tensor* t, const void* blocks, size_t nbytes);
int prim_download_f64(Session* s, Tensor* t, double* dst, size_t n);

// op nodes (nullptr on a shape / type mismatch)
Tensor* prim_binary(Session* s, int op, Tensor* a, Tensor* b);          // kOpAdd / kOpSub / kOpMul, b broadcast
Tensor* prim_scale(Session* s, Tensor* a, double v);
Tensor* prim_unary(Session* s, int op, Tensor* a, Tensor* b);           // kOpSilu, kOpSiluBack(x, dy), kOpSwiglu
Tensor* prim_mul_mat(Session* s, Tensor* a, Tensor* b);
Tensor* prim_out_prod(Session* s, Tensor* a, Tensor* b);
Tensor* prim_rms_norm(Session* s, Tensor* x, double eps);
Tensor* prim_rms_norm_back(Session* s, Tensor* x, Tensor* dy, double eps);
Tensor* prim_rope(Session* s, int op, Tensor* a, Tensor* pos, int n_dims, double base, double fscale, double ext,
                  double attn, Tensor* ff);
Tensor* prim_softmax(Session* s, Tensor* a, Tensor* mask, double scale, double max_bias);
Tensor* prim_softmax_back(Session* s, Tensor* y, Tensor* dy, double scale);
Tensor* prim_diag_mask(Session* s, int op, Tensor* a, int n_past);
Tensor* prim_permute(Session* s, Tensor* a, int p0, int p1, int p2, int p3);
Tensor* prim_reshape(Session* s, Tensor* a, int ne0, int ne1, int ne2, int ne3);
Tensor* prim_cont(Session* s, Tensor* a, int ne0, int ne1, int ne2, int ne3);
Tensor* prim_view(Session* s, Tensor* a, int ne0, int ne1, int ne2, size_t nb1, size_t nb2, size_t offset);
Tensor* prim_concat(Session* s, Tensor* a, Tensor* b, int dim);
Tensor* prim_get_rows(Session* s, Tensor* table, Tensor* idx);
Tensor* prim_mul_mat_id(Session* s, Tensor* as, Tensor* b, Tensor* ids);   // ggml_mul_mat_id (forward)
Tensor* prim_add_id(Session* s, Tensor* a, Tensor* b, Tensor* ids);        // ggml_add_id (forward)
Tensor* prim_argsort(Session* s, Tensor* a, int descending, int k);        // k = 0: argsort; k > 0: top_k
Tensor* prim_detach(Session* s, Tensor* a);                                // forward identity, no gradient
Tensor* prim_cpy(Session* s, Tensor* a, Tensor* b);                        // b's storage := a; returns b's view
Tensor* prim_set_rows(Session* s, Tensor* a, Tensor* b, Tensor* idx);      // a[idx[i]] := b[i]; returns a's view
Tensor* prim_get_rows_back(Session* s, Tensor* g, Tensor* idx, Tensor* like);
Tensor* prim_cross_entropy(Session* s, Tensor* a, Tensor* b);
Tensor* prim_sum(Session* s, int op, Tensor* a);                        // kOpSum / kOpSumRows
Tensor* prim_opt_adamw(Session* s, Tensor* a, Tensor* g, Tensor* m, Tensor* v, Tensor* hp);
Tensor* prim_opt_sgd(Session* s, Tensor* a, Tensor* g, Tensor* hp);     // hp = [alpha, wd]
Tensor* prim_cast(Session* s, Tensor* a, int type);                    // to F32: copy, or Q8_0 dequantised
// ggml_flash_attn_ext semantics (inference): q [dh, Tq, H, B], k / v [dh, Tk, KV, B],
// mask [Tk, >= Tq] or null -> [dh, H, Tq, B]; composed of score product, softmax, value product
Tensor* prim_flash_attn_ext(Session* s, Tensor* q, Tensor* k, Tensor* v, Tensor* mask, double scale, double max_bias);
int prim_upload_f32_raw(Session* s, Tensor* t, const float* src, size_t n);
int prim_download_f32_raw(Session* s, Tensor* t, float* dst, size_t n);

// programs
int prim_build_forward(Session* s, Tensor* result);
int prim_realize(Session* s, Tensor* result);
int prim_compute(Session* s);
int prim_build_backward(Session* s);
int prim_realize_backward(Session* s);
int prim_compute_backward(Session* s);

}  // namespace tb2
