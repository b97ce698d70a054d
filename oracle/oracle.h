/*
 * oracle.h — CPU restatement of the reference's TensorRegion semantics.
 *
 * TEST INFRASTRUCTURE ONLY. The engine (thiran_b200/) never links, loads or
 * calls anything in oracle/; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py do, and only as the checker or
 * the timed CPU baseline.
 *
 * Pinning: oracle/ref_driver.cpp compiles the reference's own Evaluator and
 * NativeCpu emitter from its sources (oracle/Makefile) and
 * tests/golden/make_golden.py records their outputs as fixtures; the CPU test
 * suite checks this restatement against those fixtures, against the
 * known-answer vectors of the reference's tests, and against the output
 * digests the reference recorded in its qualification run
 * (benchmarks/results/TH-023-machine.json).
 */
#ifndef THIRAN_ORACLE_H
#define THIRAN_ORACLE_H

#include <stdint.h>

#include "../include/thiran_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Evaluates a region on host values (same thb_abi_arg records the engine's
 * thb_region_execute takes, host pointers) following the reference's native
 * CPU semantics: IR-ordered, separately rounded f32 operations
 * (src/backend/v0/NativeCpu.cpp:251-316), checked i64 arithmetic
 * (NativeCpu.cpp:116-132), recipe evaluation (src/extension/v0/
 * Extension.cpp:151-169), checked index (NativeCpu.cpp:133-148). Engine ops:
 * Relu (torch.relu), Softmax / RowMax / Sum with f64 accumulation.
 * Returns 0, or 2 with the failure id (TH-SPEC-I64-OVERFLOW, TH-SPEC-BOUNDS,
 * TH021-DIVIDE-BY-ZERO) in `failure`, or 1 for a malformed call. */
int orc_region_eval(const thb_region_desc* region, const thb_abi_arg* args, uint64_t argc, void* output,
                    uint64_t output_count, char* failure, uint64_t failure_cap);

/* Scalar recipe evaluation (Extension.cpp:151-169). Returns 0 or 2
 * (divide by zero). */
int orc_recipe_eval(const thb_scalar_recipe* recipe, const float* inputs, float* result);

/* Row softmax over the last axis: m = max, e = exp(x - m) in f64, y = e / sum. */
void orc_softmax_rows(const float* x, float* y, uint64_t rows, uint64_t cols);
void orc_max_rows(const float* x, float* y, uint64_t rows, uint64_t cols);
/* Row sums accumulated in f64 and rounded once. */
void orc_sum_rows(const float* x, float* y, uint64_t rows, uint64_t cols);
void orc_sum_cols(const float* x, float* y, uint64_t rows, uint64_t cols);
/* Full sum: f64 accumulation (the 1e-5 gate) and the reference Evaluator's
 * sequential f32 order (Evaluator.cpp:221-226). */
double orc_sum_all_f64(const float* x, uint64_t n);
float orc_sum_all_sequential_f32(const float* x, uint64_t n);

/* Evaluator matmul order (src/semantic/v0/Evaluator.cpp:125-154): for each
 * (i, j), acc = 0.0f; acc = acc + a[i,k] * b[k,j] over k in order, every
 * product and sum rounded to f32. a: [m,k] row-major, b: [k,n] row-major. */
void orc_matmul_f32(const float* a, const float* b, float* c, uint64_t m, uint64_t k, uint64_t n);
/* The i64 rule (Evaluator.cpp:143-153): checked multiply and add in the same
 * order; returns 1 at the first overflow (TH-SPEC-I64-OVERFLOW), else 0. */
int orc_matmul_i64(const int64_t* a, const int64_t* b, int64_t* c, uint64_t m, uint64_t k, uint64_t n);
/* Same product accumulated in f64 and rounded once (used at sizes where the
 * sequential f32 order itself carries more error than the gate). */
void orc_matmul_f64acc(const float* a, const float* b, float* c, uint64_t m, uint64_t k, uint64_t n);

/* Rounds f32 values to bf16 (round to nearest even) and back to f32. */
void orc_round_bf16(const float* x, float* y, uint64_t n);

/* Two-layer MLP step restated from the reference's reverse-AD rules
 * (src/autodiff/v0/Autodiff.cpp:195-231) and SGD (src/training/v0/
 * Training.cpp:343-381), with the engine's precision contract: GEMM operands
 * are rounded to bf16 (X, W1, H, W2, dY, dH), products accumulate in f64.
 *   H = relu(X W1)          X [b,i], W1 [i,h]
 *   Y = H W2                W2 [h,o]
 *   L = mean((Y - T)^2)
 *   dY = 2 (Y - T) / (b*o)
 *   dW2 = H^T dY ; dH = (dY W2^T) * [H > 0] ; dW1 = X^T dH
 *   W1 -= lr dW1 ; W2 -= lr dW2
 * Outputs: loss, dW1 [i,h], dW2 [h,o], updated W1/W2 in place. */
double orc_mlp_step(const float* x, const float* t, float* w1, float* w2, uint64_t b, uint64_t i, uint64_t h,
                    uint64_t o, float lr, float* dw1, float* dw2, float* hidden, float* y);

/* One optimizer update of n parameters (src/training/v0/Training.cpp:366-372):
 * with a velocity v, d = v*mu + g and v = d (SGDMomentum); without, d = g
 * (SGD); then p = p - d*lr. Each operation rounds to f32. */
void orc_sgd_update(float* p, const float* g, float* v, float mu, float lr, uint64_t n);

/* FNV-1a over the little-endian bytes of n f32 bit patterns, starting from
 * `basis`: the reference's output digests (benchmarks/th023/
 * Qualification.cpp:176-187 starts from 1469598103934665603,
 * src/graphics/v0/Graphics.cpp:188-200 from 14695981039346656037). */
uint64_t orc_fnv1a64_f32(const float* values, uint64_t n, uint64_t basis);

/* The same step with the optional parts of the examples/mlp.th structure and
 * the reference optimizer:
 *   biases (b1 [h], b2 [o], broadcast over rows, Evaluator.cpp:95-124):
 *     H = relu(X W1 + b1), Y = H W2 + b2; their gradients are the column sums
 *     of dH and dY (reduceToShape, Evaluator.cpp:258-277; f64 accumulation);
 *   SGD with momentum mu (Training.cpp:366-372): d = v*mu + g; v = d;
 *     p = p - d*lr, for every parameter (W1, b1, W2, b2).
 * NULL b1/b2 = no biases; momentum 0 with NULL velocities = plain SGD. */
typedef struct {
    float* b1;        /* [h], updated in place */
    float* b2;        /* [o], updated in place */
    float momentum;
    float* v_w1;      /* velocities, same shapes, updated in place */
    float* v_b1;
    float* v_w2;
    float* v_b2;
    float* db1;       /* out: bias gradients (optional) */
    float* db2;
} orc_mlp_extras;

double orc_mlp_step_ex(const float* x, const float* t, float* w1, float* w2, uint64_t b, uint64_t i, uint64_t h,
                       uint64_t o, float lr, float* dw1, float* dw2, float* hidden, float* y,
                       const orc_mlp_extras* extras);

/* ---- software renderer (src/graphics/v0/Graphics.cpp) ----------------------
 * Matrices are 16 f32, row-major, column-vector convention (P*V*M). Every f32
 * product and sum is rounded separately, as the reference's volatile helpers
 * do; the rasterizer works in f64 without contraction. Returns 0 or a
 * TH019-* failure id (static string). */
void orc_gfx_identity(float* m);
void orc_gfx_rotation_x(float radians, float* m);
void orc_gfx_rotation_y(float radians, float* m);
void orc_gfx_rotation_z(float radians, float* m);
void orc_gfx_translation(float x, float y, float z, float* m);
void orc_gfx_scale(float x, float y, float z, float* m);
void orc_gfx_multiply(const float* a, const float* b, float* out);
const char* orc_gfx_look_at(const float* eye, const float* target, const float* up, float* m);
const char* orc_gfx_perspective(float fovy, float aspect, float near_distance, float far_distance, float* m);
const char* orc_gfx_orthographic(float left, float right, float bottom, float top, float near_distance,
                                 float far_distance, float* m);
/* render(): color [w*h][4] and depth [w*h] outputs; stats = input triangles,
 * post-clip triangles, shaded pixels, depth passes. */
const char* orc_render(const float* positions, uint64_t vertices, const int64_t* indices, uint64_t triangles,
                       const float* colors, const float* model, const float* view, const float* projection,
                       uint64_t width, uint64_t height, const float* clear, float* color, float* depth,
                       uint64_t* stats);

#ifdef __cplusplus
}
#endif

#endif
