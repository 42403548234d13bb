/*
 * anelm oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * Builds the layer glue of oracle/glue_impl.h on top of the reference's OWN
 * core/cpu_ops.cpp (compiled unmodified by oracle/Makefile, against the
 * Accelerate stand-in in oracle/shim/).  The result, oracle/_ref/libref_core.so,
 * is the reference CPU attention core run on this machine: it pins the C
 * restatement (liboracle.so), generates the golden fixtures in tests/golden/,
 * and is the CPU baseline bench.py times.
 *
 * Exported names: ref_<op> for each cpu_ops.h entry point (core/cpu_ops.h:16-58)
 * and ref_<glue> for the glue functions.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "cpu_ops.h"      /* the reference header, core/cpu_ops.h */
#include "anelm_oracle.h" /* orc_shape / orc_variant */

#define OP(name) ane_lm::name
#define GLUE(name) ref_##name

extern "C" {

#include "glue_impl.h"

void ref_silu_vec_inplace(float* x, int n, float* tmp) { ane_lm::silu_vec_inplace(x, n, tmp); }
void ref_mul_sigmoid_inplace(float* y, const float* z, int n, float* tmp) {
    ane_lm::mul_sigmoid_inplace(y, z, n, tmp);
}
void ref_rmsnorm(float* out, const float* x, const float* w, int dim, float eps) {
    ane_lm::rmsnorm(out, x, w, dim, eps);
}
void ref_rmsnorm_gated(float* out, const float* x, const float* z, const float* w, int dim) {
    ane_lm::rmsnorm_gated(out, x, z, w, dim);
}
void ref_apply_rope_cached(float* q, float* k, int nq, int nkv, int hd, int qs, int ks, int rot,
                           int pos, float theta, const float* c, const float* s) {
    ane_lm::apply_rope_cached(q, k, nq, nkv, hd, qs, ks, rot, pos, theta, c, s);
}
void ref_softmax(float* x, int n) { ane_lm::softmax(x, n); }
void ref_matvec(float* y, const float* W, const float* x, int o, int i) { ane_lm::matvec(y, W, x, o, i); }
void ref_l2_normalize(float* x, int dim) { ane_lm::l2_normalize(x, dim); }
void ref_conv1d_update(float* y, float* st, int* pos, const float* x, const float* w, int c, int k) {
    ane_lm::conv1d_update(y, st, pos, x, w, c, k);
}
void ref_ssm_step(float* y, float* state, const float* q, const float* k, const float* v,
                  float decay, float beta, int kd, int vd) {
    ane_lm::ssm_step(y, state, q, k, v, decay, beta, kd, vd);
}
void ref_gqa_attention(float* out, const float* q, const float* kc, const float* vc, int nh, int nkv,
                       int hd, int qs, int start, int len, int cap) {
    ane_lm::gqa_attention(out, q, kc, vc, nh, nkv, hd, qs, start, len, cap);
}

}  /* extern "C" */
