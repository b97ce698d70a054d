/*
 * oracle.c — CPU restatement of the reference's TensorRegion semantics.
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Built with -ffp-contract=off so
 * every f32 expression below is one IEEE-rounded operation, like the
 * reference's `volatile float` temporaries (src/backend/v0/NativeCpu.cpp:287).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int tensor;
    uint32_t dtype;
    uint32_t rank;
    uint64_t shape[2];
    uint64_t count;
    void* data; /* tensor elements */
    int owned;
    int64_t i;
    float f;
} value_t;

static void set_failure(char* out, uint64_t cap, const char* text) {
    if (!out || cap == 0) return;
    size_t n = strlen(text);
    if (n > cap - 1) n = (size_t)(cap - 1);
    memcpy(out, text, n);
    out[n] = '\0';
}

static int position_of(const thb_region_desc* r, uint32_t id) {
    for (uint32_t p = 0; p < r->node_count; ++p)
        if (r->nodes[p].id == id) return (int)p;
    return -1;
}

/* Checked i64 arithmetic: fails exactly when the mathematical result leaves
 * [INT64_MIN, INT64_MAX] (checked_add/sub/mul/neg, NativeCpu.cpp:116-132). */
static int checked(int op, int64_t a, int64_t b, int64_t* r) {
    switch (op) {
    case THB_OP_ADD: return __builtin_add_overflow(a, b, r);
    case THB_OP_SUBTRACT: return __builtin_sub_overflow(a, b, r);
    case THB_OP_ELEMENT_MULTIPLY: return __builtin_mul_overflow(a, b, r);
    case THB_OP_NEGATE:
        if (a == INT64_MIN) return 1;
        *r = -a;
        return 0;
    }
    return 1;
}

int orc_recipe_eval(const thb_scalar_recipe* recipe, const float* inputs, float* result) {
    float values[256];
    if (!recipe || recipe->node_count == 0 || recipe->node_count > 256) return 1;
    for (size_t k = 0; k < recipe->node_count; ++k) {
        const thb_scalar_node* n = &recipe->nodes[k];
        switch (n->opcode) {
        case THB_SCALAR_INPUT: values[k] = inputs[n->input]; break;
        case THB_SCALAR_CONSTANT_F32: values[k] = n->constant; break;
        case THB_SCALAR_ADD: values[k] = values[n->left] + values[n->right]; break;
        case THB_SCALAR_SUBTRACT: values[k] = values[n->left] - values[n->right]; break;
        case THB_SCALAR_MULTIPLY: values[k] = values[n->left] * values[n->right]; break;
        case THB_SCALAR_DIVIDE:
            if (values[n->right] == 0.0f) return 2;
            values[k] = values[n->left] / values[n->right];
            break;
        case THB_SCALAR_NEGATE: values[k] = -values[n->left]; break;
        default: return 1;
        }
    }
    *result = values[recipe->root];
    return 0;
}

static float relu(float x) { return (x > 0.0f || x != x) ? x : 0.0f; }

void orc_softmax_rows(const float* x, float* y, uint64_t rows, uint64_t cols) {
    double* e = (double*)malloc(sizeof(double) * (cols ? cols : 1));
    for (uint64_t r = 0; r < rows; ++r) {
        const float* in = x + r * cols;
        float m = -INFINITY;
        for (uint64_t j = 0; j < cols; ++j) m = in[j] > m ? in[j] : m;
        double s = 0.0;
        for (uint64_t j = 0; j < cols; ++j) {
            e[j] = exp((double)in[j] - (double)m);
            s += e[j];
        }
        for (uint64_t j = 0; j < cols; ++j) y[r * cols + j] = (float)(e[j] / s);
    }
    free(e);
}

void orc_max_rows(const float* x, float* y, uint64_t rows, uint64_t cols) {
    for (uint64_t r = 0; r < rows; ++r) {
        float m = -INFINITY;
        for (uint64_t j = 0; j < cols; ++j) m = x[r * cols + j] > m ? x[r * cols + j] : m;
        y[r] = m;
    }
}

void orc_sum_rows(const float* x, float* y, uint64_t rows, uint64_t cols) {
    for (uint64_t r = 0; r < rows; ++r) {
        double s = 0.0;
        for (uint64_t j = 0; j < cols; ++j) s += x[r * cols + j];
        y[r] = (float)s;
    }
}

void orc_sum_cols(const float* x, float* y, uint64_t rows, uint64_t cols) {
    double* s = (double*)calloc(cols ? cols : 1, sizeof(double));
    for (uint64_t r = 0; r < rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) s[c] += x[r * cols + c];
    for (uint64_t c = 0; c < cols; ++c) y[c] = (float)s[c];
    free(s);
}

double orc_sum_all_f64(const float* x, uint64_t n) {
    double s = 0.0;
    for (uint64_t k = 0; k < n; ++k) s += x[k];
    return s;
}

float orc_sum_all_sequential_f32(const float* x, uint64_t n) {
    float acc = 0.0f;
    for (uint64_t k = 0; k < n; ++k) acc = acc + x[k];
    return acc;
}

void orc_matmul_f32(const float* a, const float* b, float* c, uint64_t m, uint64_t k, uint64_t n) {
    for (uint64_t i = 0; i < m; ++i)
        for (uint64_t j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (uint64_t p = 0; p < k; ++p) {
                const float product = a[i * k + p] * b[p * n + j];
                acc = acc + product;
            }
            c[i * n + j] = acc;
        }
}

int orc_matmul_i64(const int64_t* a, const int64_t* b, int64_t* c, uint64_t m, uint64_t k, uint64_t n) {
    /* Evaluator.cpp:143-153: acc = checked(acc + checked(a * b)), k in order;
     * returns 1 at the first overflow (the reference fails there). */
    for (uint64_t i = 0; i < m; ++i)
        for (uint64_t j = 0; j < n; ++j) {
            int64_t acc = 0;
            for (uint64_t p = 0; p < k; ++p) {
                int64_t product;
                if (__builtin_mul_overflow(a[i * k + p], b[p * n + j], &product)) return 1;
                if (__builtin_add_overflow(acc, product, &acc)) return 1;
            }
            c[i * n + j] = acc;
        }
    return 0;
}

void orc_matmul_f64acc(const float* a, const float* b, float* c, uint64_t m, uint64_t k, uint64_t n) {
    double* row = (double*)malloc(sizeof(double) * (n ? n : 1));
    for (uint64_t i = 0; i < m; ++i) {
        for (uint64_t j = 0; j < n; ++j) row[j] = 0.0;
        for (uint64_t p = 0; p < k; ++p) {
            const double av = a[i * k + p];
            const float* br = b + p * n;
            for (uint64_t j = 0; j < n; ++j) row[j] += av * (double)br[j];
        }
        for (uint64_t j = 0; j < n; ++j) c[i * n + j] = (float)row[j];
    }
    free(row);
}

void orc_round_bf16(const float* x, float* y, uint64_t n) {
    for (uint64_t k = 0; k < n; ++k) {
        uint32_t bits;
        memcpy(&bits, &x[k], 4);
        if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu)) {
            bits |= 0x00400000u; /* quiet NaN */
        } else {
            const uint32_t lsb = (bits >> 16) & 1u;
            bits += 0x7fffu + lsb;
        }
        bits &= 0xffff0000u;
        memcpy(&y[k], &bits, 4);
    }
}

static void transpose(const float* x, float* y, uint64_t rows, uint64_t cols) {
    for (uint64_t r = 0; r < rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) y[c * rows + r] = x[r * cols + c];
}

double orc_mlp_step(const float* x, const float* t, float* w1, float* w2, uint64_t b, uint64_t i, uint64_t h,
                    uint64_t o, float lr, float* dw1, float* dw2, float* hidden, float* yout) {
    return orc_mlp_step_ex(x, t, w1, w2, b, i, h, o, lr, dw1, dw2, hidden, yout, NULL);
}

/* Column sums of a [rows, cols] matrix, f64 accumulation in row order. */
static void column_sums(const float* m, float* out, uint64_t rows, uint64_t cols) {
    for (uint64_t c = 0; c < cols; ++c) {
        double acc = 0.0;
        for (uint64_t r = 0; r < rows; ++r) acc += (double)m[r * cols + c];
        out[c] = (float)acc;
    }
}

uint64_t orc_fnv1a64_f32(const float* values, uint64_t n, uint64_t basis) {
    uint64_t hash = basis;
    for (uint64_t k = 0; k < n; ++k) {
        uint32_t bits;
        memcpy(&bits, &values[k], 4);
        for (unsigned shift = 0; shift < 32; shift += 8) {
            hash ^= (uint8_t)(bits >> shift);
            hash *= 1099511628211ULL;
        }
    }
    return hash;
}

void orc_sgd_update(float* p, const float* g, float* v, float mu, float lr, uint64_t n) {
    for (uint64_t k = 0; k < n; ++k) {
        float d = g[k];
        if (v) {
            const float scaled = v[k] * mu;
            d = scaled + g[k];
            v[k] = d;
        }
        const float step = d * lr;
        p[k] = p[k] - step;
    }
}

double orc_mlp_step_ex(const float* x, const float* t, float* w1, float* w2, uint64_t b, uint64_t i, uint64_t h,
                       uint64_t o, float lr, float* dw1, float* dw2, float* hidden, float* yout,
                       const orc_mlp_extras* ex) {
    const orc_mlp_extras none = {0};
    if (!ex) ex = &none;
    float* xb = (float*)malloc(sizeof(float) * b * i);
    float* w1b = (float*)malloc(sizeof(float) * i * h);
    float* w2b = (float*)malloc(sizeof(float) * h * o);
    float* hb = (float*)malloc(sizeof(float) * b * h);
    float* y = (float*)malloc(sizeof(float) * b * o);
    float* dy = (float*)malloc(sizeof(float) * b * o);
    float* dyb = (float*)malloc(sizeof(float) * b * o);
    float* dh = (float*)malloc(sizeof(float) * b * h);
    float* tmp = (float*)malloc(sizeof(float) * (b * h > h * o ? (b * h > i * b ? b * h : i * b) : (h * o > i * b ? h * o : i * b)));
    float* tr = (float*)malloc(sizeof(float) * (b * h > b * i ? b * h : b * i) + sizeof(float) * h * o);
    orc_round_bf16(x, xb, b * i);
    orc_round_bf16(w1, w1b, i * h);
    orc_round_bf16(w2, w2b, h * o);
    /* forward */
    orc_matmul_f64acc(xb, w1b, hidden, b, i, h);
    if (ex->b1)
        for (uint64_t k = 0; k < b * h; ++k) hidden[k] = hidden[k] + ex->b1[k % h];
    for (uint64_t k = 0; k < b * h; ++k) hidden[k] = relu(hidden[k]);
    orc_round_bf16(hidden, hb, b * h);
    orc_matmul_f64acc(hb, w2b, y, b, h, o);
    if (ex->b2)
        for (uint64_t k = 0; k < b * o; ++k) y[k] = y[k] + ex->b2[k % o];
    double loss = 0.0;
    const float scale = 2.0f / (float)(b * o);
    for (uint64_t k = 0; k < b * o; ++k) {
        const float d = y[k] - t[k];
        loss += (double)d * (double)d;
        dy[k] = d * scale;
    }
    loss /= (double)(b * o);
    float* db1 = (float*)malloc(sizeof(float) * h);
    float* db2 = (float*)malloc(sizeof(float) * o);
    if (ex->b2) column_sums(dy, db2, b, o);
    orc_round_bf16(dy, dyb, b * o);
    /* backward: dW2 = H^T dY */
    transpose(hb, tr, b, h);
    orc_matmul_f64acc(tr, dyb, dw2, h, b, o);
    /* dH = (dY W2^T) * [H > 0] */
    transpose(w2b, tmp, h, o);
    orc_matmul_f64acc(dyb, tmp, dh, b, o, h);
    for (uint64_t k = 0; k < b * h; ++k) dh[k] = hidden[k] > 0.0f ? dh[k] : 0.0f;
    if (ex->b1) column_sums(dh, db1, b, h);
    orc_round_bf16(dh, dh, b * h);
    /* dW1 = X^T dH */
    transpose(xb, tr, b, i);
    orc_matmul_f64acc(tr, dh, dw1, i, b, h);
    /* Optimizer (Training.cpp:366-372), parameters in W1, b1, W2, b2 order. */
    const float mu = ex->momentum;
    orc_sgd_update(w1, dw1, ex->v_w1, mu, lr, i * h);
    if (ex->b1) orc_sgd_update(ex->b1, db1, ex->v_b1, mu, lr, h);
    orc_sgd_update(w2, dw2, ex->v_w2, mu, lr, h * o);
    if (ex->b2) orc_sgd_update(ex->b2, db2, ex->v_b2, mu, lr, o);
    if (ex->db1 && ex->b1) memcpy(ex->db1, db1, sizeof(float) * h);
    if (ex->db2 && ex->b2) memcpy(ex->db2, db2, sizeof(float) * o);
    if (yout) memcpy(yout, y, sizeof(float) * b * o);
    free(xb); free(w1b); free(w2b); free(hb); free(y); free(dy); free(dyb); free(dh); free(tmp); free(tr);
    free(db1); free(db2);
    return loss;
}

/* ---- region interpreter ------------------------------------------------------------- */

static int elementwise_op(uint32_t op) {
    return op == THB_OP_NEGATE || op == THB_OP_ADD || op == THB_OP_SUBTRACT || op == THB_OP_ELEMENT_MULTIPLY ||
           op == THB_OP_EXTENSION || op == THB_OP_RELU || op == THB_OP_EXTENSION_GRADIENT;
}

/* The recipe an Extension / ExtensionGradient node evaluates: the forward
 * recipe, or gradient recipe `axis` over (primals..., result, cotangent)
 * (src/autodiff/v0/Autodiff.cpp:231-270). */
static const thb_scalar_recipe* node_recipe(const thb_region_node* n) {
    if (n->op == THB_OP_EXTENSION) return &n->extension->forward;
    return &n->extension->derivative->gradients[n->axis];
}

int orc_region_eval(const thb_region_desc* r, const thb_abi_arg* args, uint64_t argc, void* output,
                    uint64_t output_count, char* failure, uint64_t cap) {
    int status = 0;
    value_t* vals = (value_t*)calloc(r->node_count ? r->node_count : 1, sizeof(value_t));
    if (argc != r->input_count) {
        set_failure(failure, cap, "GPU-INPUT-ARITY");
        free(vals);
        return 1;
    }
    for (uint32_t p = 0; p < r->node_count && status == 0; ++p) {
        const thb_region_node* n = &r->nodes[p];
        value_t* v = &vals[p];
        v->dtype = n->dtype;
        v->rank = n->rank;
        v->tensor = n->rank > 0;
        const value_t* d0 = n->dependency_count ? &vals[position_of(r, n->dependencies[0])] : NULL;
        if (n->op == THB_OP_INPUT) {
            uint32_t k = 0;
            while (k < r->input_count && r->inputs[k] != n->id) ++k;
            const thb_abi_arg* a = &args[k];
            if (v->tensor) {
                v->count = 1;
                for (uint32_t d = 0; d < n->rank; ++d) {
                    v->shape[d] = a->shape[d];
                    v->count *= a->shape[d];
                }
                v->data = (void*)a->data;
            } else if (n->dtype == THB_DTYPE_I64) {
                memcpy(&v->i, a->data, 8);
            } else {
                memcpy(&v->f, a->data, 4);
            }
            continue;
        }
        switch (n->op) {
        case THB_OP_INTEGER: v->i = n->integer; break;
        case THB_OP_FLOAT: v->f = n->floating; break;
        case THB_OP_ALIAS: *v = *d0; v->owned = 0; break;
        case THB_OP_TENSOR_LITERAL: {
            const size_t w = n->dtype == THB_DTYPE_I64 ? 8 : 4;
            v->count = n->dependency_count;
            for (uint32_t d = 0; d < n->rank; ++d) v->shape[d] = (uint64_t)n->extent[d];
            v->data = malloc(w * (v->count ? v->count : 1));
            v->owned = 1;
            for (uint32_t k = 0; k < n->dependency_count; ++k) {
                const value_t* s = &vals[position_of(r, n->dependencies[k])];
                if (n->dtype == THB_DTYPE_I64) ((int64_t*)v->data)[k] = s->i;
                else ((float*)v->data)[k] = s->f;
            }
            break;
        }
        case THB_OP_COPY: {
            const size_t w = n->dtype == THB_DTYPE_I64 ? 8 : 4;
            *v = *d0;
            v->data = malloc(w * (v->count ? v->count : 1));
            v->owned = 1;
            memcpy(v->data, d0->data, w * v->count);
            break;
        }
        case THB_OP_INDEX: {
            uint64_t linear = 0;
            for (uint32_t a = 0; a < n->index_count; ++a) {
                const int64_t c = vals[position_of(r, n->indices[a])].i;
                if (c < 0 || (uint64_t)c >= d0->shape[a]) {
                    set_failure(failure, cap, "TH-SPEC-BOUNDS");
                    status = 2;
                    break;
                }
                linear = linear * d0->shape[a] + (uint64_t)c;
            }
            if (status == 0) {
                if (n->dtype == THB_DTYPE_I64) v->i = ((const int64_t*)d0->data)[linear];
                else v->f = ((const float*)d0->data)[linear];
            }
            break;
        }
        case THB_OP_TRANSPOSE: {
            /* Evaluator.cpp:200-213 */
            const size_t w = n->dtype == THB_DTYPE_I64 ? 8 : 4;
            v->shape[0] = d0->shape[1];
            v->shape[1] = d0->shape[0];
            v->count = d0->count;
            v->data = malloc(w * (v->count ? v->count : 1));
            v->owned = 1;
            for (uint64_t i = 0; i < d0->shape[0]; ++i)
                for (uint64_t j = 0; j < d0->shape[1]; ++j)
                    memcpy((char*)v->data + (j * d0->shape[0] + i) * w, (const char*)d0->data + (i * d0->shape[1] + j) * w, w);
            break;
        }
        case THB_OP_MATMUL: {
            /* Evaluator.cpp:125-154: sequential-k f32, each op rounded; i64
             * with checked multiply and add (any overflow fails the call) */
            const value_t* d1 = &vals[position_of(r, n->dependencies[1])];
            v->shape[0] = d0->shape[0];
            v->shape[1] = d1->shape[1];
            v->count = v->shape[0] * v->shape[1];
            v->data = malloc(8 * (v->count ? v->count : 1));
            v->owned = 1;
            if (n->dtype == THB_DTYPE_I64) {
                if (orc_matmul_i64((const int64_t*)d0->data, (const int64_t*)d1->data, (int64_t*)v->data,
                                   d0->shape[0], d0->shape[1], d1->shape[1])) {
                    set_failure(failure, cap, "TH-SPEC-I64-OVERFLOW");
                    status = 2;
                }
            } else {
                orc_matmul_f32((const float*)d0->data, (const float*)d1->data, (float*)v->data, d0->shape[0],
                               d0->shape[1], d1->shape[1]);
            }
            break;
        }
        case THB_OP_BROADCAST_TO_SHAPE: {
            /* Evaluator.cpp:278-309: target = reference shape, source = target without `axis` */
            const value_t* ref = &vals[position_of(r, n->dependencies[1])];
            v->shape[0] = ref->shape[0];
            v->shape[1] = ref->shape[1];
            v->count = ref->count;
            v->data = malloc(4 * (v->count ? v->count : 1));
            v->owned = 1;
            for (uint64_t k = 0; k < v->count; ++k) {
                float x;
                if (!d0->tensor) x = d0->f;
                else if (ref->rank == 2) x = ((const float*)d0->data)[n->axis == 0 ? k % ref->shape[1] : k / ref->shape[1]];
                else x = ((const float*)d0->data)[0];
                ((float*)v->data)[k] = x;
            }
            break;
        }
        case THB_OP_REDUCE_TO_SHAPE: {
            /* Evaluator.cpp:258-277: sequential f32 accumulation in source order */
            const value_t* ref = &vals[position_of(r, n->dependencies[1])];
            if (!ref->tensor) {
                float acc = 0.0f;
                for (uint64_t k = 0; k < d0->count; ++k) acc = acc + ((const float*)d0->data)[k];
                v->f = acc;
                v->tensor = 0;
                break;
            }
            v->shape[0] = ref->shape[0];
            v->shape[1] = ref->shape[1];
            v->count = ref->count;
            v->data = calloc(v->count ? v->count : 1, 4);
            v->owned = 1;
            const uint32_t delta = d0->rank - ref->rank;
            for (uint64_t k = 0; k < d0->count; ++k) {
                uint64_t sc[2] = {0, 0}, tc[2] = {0, 0};
                if (d0->rank == 2) { sc[0] = k / d0->shape[1]; sc[1] = k % d0->shape[1]; }
                else sc[0] = k;
                for (uint32_t d = 0; d < ref->rank; ++d) tc[d] = ref->shape[d] == 1 ? 0 : sc[d + delta];
                const uint64_t t = ref->rank == 2 ? tc[0] * ref->shape[1] + tc[1] : tc[0];
                ((float*)v->data)[t] = ((float*)v->data)[t] + ((const float*)d0->data)[k];
            }
            break;
        }
        case THB_OP_ZERO_LIKE:
            v->shape[0] = d0->shape[0];
            v->shape[1] = d0->shape[1];
            v->count = d0->count;
            v->data = calloc(v->count ? v->count : 1, 4);
            v->owned = 1;
            break;
        case THB_OP_SUM:
            if (n->dtype == THB_DTYPE_I64) {
                /* Evaluator.cpp:237-250: acc = checked(acc + v) in order */
                const uint64_t rows = d0->rank == 2 ? d0->shape[0] : 1;
                const uint64_t cols = d0->rank == 2 ? d0->shape[1] : d0->shape[0];
                const int64_t* x = (const int64_t*)d0->data;
                const uint64_t outer = n->rank == 0 ? 1 : (n->axis == 1 ? rows : cols);
                const uint64_t inner = n->rank == 0 ? d0->count : (n->axis == 1 ? cols : rows);
                v->count = n->rank == 0 ? 1 : outer;
                v->shape[0] = outer;
                v->data = malloc(8 * (v->count ? v->count : 1));
                v->owned = 1;
                for (uint64_t o = 0; o < outer && status == 0; ++o) {
                    int64_t acc = 0;
                    for (uint64_t k = 0; k < inner; ++k) {
                        const int64_t e = n->rank == 0 ? x[k] : (n->axis == 1 ? x[o * cols + k] : x[k * cols + o]);
                        if (__builtin_add_overflow(acc, e, &acc)) {
                            set_failure(failure, cap, "TH-SPEC-I64-OVERFLOW");
                            status = 2;
                            break;
                        }
                    }
                    if (n->rank == 0) v->i = acc;
                    else ((int64_t*)v->data)[o] = acc;
                }
                break;
            }
            /* fall through: f32 sums */
        case THB_OP_SOFTMAX: case THB_OP_ROW_MAX: {
            const uint64_t rows = d0->rank == 2 ? d0->shape[0] : 1;
            const uint64_t cols = d0->rank == 2 ? d0->shape[1] : d0->shape[0];
            v->count = 1;
            if (n->op == THB_OP_SOFTMAX) {
                v->shape[0] = d0->shape[0];
                v->shape[1] = d0->shape[1];
                v->count = d0->count;
            } else if (n->rank == 1) {
                v->shape[0] = (n->op == THB_OP_SUM && n->axis == 0) ? cols : rows;
                v->count = v->shape[0];
            }
            v->data = malloc(4 * (v->count ? v->count : 1));
            v->owned = 1;
            if (n->op == THB_OP_SOFTMAX) orc_softmax_rows((const float*)d0->data, (float*)v->data, rows, cols);
            else if (n->op == THB_OP_ROW_MAX) orc_max_rows((const float*)d0->data, (float*)v->data, rows, cols);
            else if (n->rank == 0) v->f = (float)orc_sum_all_f64((const float*)d0->data, d0->count);
            else if (n->axis == 1) orc_sum_rows((const float*)d0->data, (float*)v->data, rows, cols);
            else orc_sum_cols((const float*)d0->data, (float*)v->data, rows, cols);
            break;
        }
        default:
            if (!elementwise_op(n->op)) {
                set_failure(failure, cap, "GPU-UNSUPPORTED-OP");
                status = 1;
                break;
            }
            {
                /* Scalar operands broadcast (Evaluator.cpp:95-124): the
                 * result takes the tensor operand's shape. */
                const value_t* d1 = n->dependency_count > 1 ? &vals[position_of(r, n->dependencies[1])] : NULL;
                *v = (d0->tensor || !d1) ? *d0 : *d1;
            }
            v->dtype = n->dtype;
            v->data = malloc((n->dtype == THB_DTYPE_I64 ? 8 : 4) * (v->count ? v->count : 1));
            v->owned = 1;
            for (uint64_t k = 0; k < v->count && status == 0; ++k) {
                const value_t* d1 = n->dependency_count > 1 ? &vals[position_of(r, n->dependencies[1])] : NULL;
                if (n->dtype == THB_DTYPE_I64) {
                    const int64_t a = d0->tensor ? ((const int64_t*)d0->data)[k] : d0->i;
                    int64_t b = 0, out = 0;
                    if (d1) b = d1->tensor ? ((const int64_t*)d1->data)[k] : d1->i;
                    if (checked((int)n->op, a, b, &out)) {
                        set_failure(failure, cap, "TH-SPEC-I64-OVERFLOW");
                        status = 2;
                    }
                    ((int64_t*)v->data)[k] = out;
                } else {
                    const float a = d0->tensor ? ((const float*)d0->data)[k] : d0->f;
                    float out = 0.0f;
                    if (n->op == THB_OP_EXTENSION || n->op == THB_OP_EXTENSION_GRADIENT) {
                        float in[10];
                        for (uint32_t j = 0; j < n->dependency_count && j < 10; ++j)
                            in[j] = ((const float*)vals[position_of(r, n->dependencies[j])].data)[k];
                        const int rs = orc_recipe_eval(node_recipe(n), in, &out);
                        if (rs == 2) {
                            set_failure(failure, cap, "TH021-DIVIDE-BY-ZERO");
                            status = 2;
                        } else if (rs) {
                            set_failure(failure, cap, "TRV11");
                            status = 1;
                        }
                    } else if (n->op == THB_OP_NEGATE) {
                        out = -a;
                    } else if (n->op == THB_OP_RELU) {
                        out = relu(a);
                    } else {
                        const float b = d1->tensor ? ((const float*)d1->data)[k] : d1->f;
                        out = n->op == THB_OP_ADD ? a + b : n->op == THB_OP_SUBTRACT ? a - b : a * b;
                    }
                    ((float*)v->data)[k] = out;
                }
            }
            break;
        }
    }
    if (status == 0) {
        const value_t* out = &vals[position_of(r, r->output)];
        const size_t w = out->dtype == THB_DTYPE_I64 ? 8 : 4;
        if (out->tensor) {
            if (output_count != out->count) {
                set_failure(failure, cap, "GPU-OUTPUT-SHAPE");
                status = 1;
            } else if (out->count) {
                memcpy(output, out->data, w * out->count);
            }
        } else if (output_count != 1) {
            set_failure(failure, cap, "GPU-OUTPUT-SHAPE");
            status = 1;
        } else if (out->dtype == THB_DTYPE_I64) {
            memcpy(output, &out->i, 8);
        } else {
            memcpy(output, &out->f, 4);
        }
    }
    for (uint32_t p = 0; p < r->node_count; ++p)
        if (vals[p].owned) free(vals[p].data);
    free(vals);
    return status;
}

/* ---- software renderer ------------------------------------------------------------
 * Restatement of src/graphics/v0/Graphics.cpp. This file is compiled with
 * -ffp-contract=off, so each f32 / f64 operation below rounds on its own like
 * the reference's volatile helpers (:22-41). */

static int gfx_finite(float v) { return isfinite(v); }

static void gfx_set(float* m, const float* v) { memcpy(m, v, 16 * sizeof(float)); }

void orc_gfx_identity(float* m) {
    const float v[16] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1};
    gfx_set(m, v);
}

void orc_gfx_translation(float x, float y, float z, float* m) {
    const float v[16] = {1, 0, 0, x, 0, 1, 0, y, 0, 0, 1, z, 0, 0, 0, 1};
    gfx_set(m, v);
}

void orc_gfx_scale(float x, float y, float z, float* m) {
    const float v[16] = {x, 0, 0, 0, 0, y, 0, 0, 0, 0, z, 0, 0, 0, 0, 1};
    gfx_set(m, v);
}

/* Graphics.cpp:448-473 (cosf / sinf of the host C library). */
void orc_gfx_rotation_x(float r, float* m) {
    const float c = cosf(r), s = sinf(r);
    const float v[16] = {1, 0, 0, 0, 0, c, -s, 0, 0, s, c, 0, 0, 0, 0, 1};
    gfx_set(m, v);
}

void orc_gfx_rotation_y(float r, float* m) {
    const float c = cosf(r), s = sinf(r);
    const float v[16] = {c, 0, s, 0, 0, 1, 0, 0, -s, 0, c, 0, 0, 0, 0, 1};
    gfx_set(m, v);
}

void orc_gfx_rotation_z(float r, float* m) {
    const float c = cosf(r), s = sinf(r);
    const float v[16] = {c, -s, 0, 0, s, c, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1};
    gfx_set(m, v);
}

/* multiply (:475-485): out[r][c] accumulates a[r][k]*b[k][c] over k from 0.0f. */
void orc_gfx_multiply(const float* a, const float* b, float* out) {
    float r[16];
    for (int row = 0; row < 4; ++row)
        for (int col = 0; col < 4; ++col) {
            float acc = 0.0f;
            for (int k = 0; k < 4; ++k) {
                const float p = a[row * 4 + k] * b[k * 4 + col];
                acc = acc + p;
            }
            r[row * 4 + col] = acc;
        }
    gfx_set(out, r);
}

static float gfx_dot(const float* a, const float* b) {
    float acc = 0.0f;
    for (int k = 0; k < 3; ++k) {
        const float p = a[k] * b[k];
        acc = acc + p;
    }
    return acc;
}

static void gfx_cross(const float* a, const float* b, float* out) {
    const float x1 = a[1] * b[2], x2 = a[2] * b[1];
    const float y1 = a[2] * b[0], y2 = a[0] * b[2];
    const float z1 = a[0] * b[1], z2 = a[1] * b[0];
    out[0] = x1 + -x2;
    out[1] = y1 + -y2;
    out[2] = z1 + -z2;
}

static int gfx_normalize(const float* v, float* out) {
    const float len2 = gfx_dot(v, v);
    if (!gfx_finite(len2) || len2 <= 0.0f) return 0;
    const float len = sqrtf(len2);
    if (!gfx_finite(len) || len <= 1.1920928955078125e-07f) return 0;
    for (int k = 0; k < 3; ++k) {
        out[k] = v[k] / len;
        if (!gfx_finite(out[k])) return 0;
    }
    return 1;
}

/* lookAt (:499-512). */
const char* orc_gfx_look_at(const float* eye, const float* target, const float* up, float* m) {
    for (int k = 0; k < 3; ++k)
        if (!gfx_finite(eye[k]) || !gfx_finite(target[k]) || !gfx_finite(up[k])) return "TH019-CAMERA";
    float dir[3] = {target[0] - eye[0], target[1] - eye[1], target[2] - eye[2]};
    float forward[3], sideRaw[3], side[3], cameraUp[3];
    if (!gfx_normalize(dir, forward)) return "TH019-CAMERA-DIRECTION";
    gfx_cross(forward, up, sideRaw);
    if (!gfx_normalize(sideRaw, side)) return "TH019-CAMERA-UP";
    gfx_cross(side, forward, cameraUp);
    const float v[16] = {side[0], side[1], side[2], -gfx_dot(side, eye),
                         cameraUp[0], cameraUp[1], cameraUp[2], -gfx_dot(cameraUp, eye),
                         -forward[0], -forward[1], -forward[2], gfx_dot(forward, eye),
                         0, 0, 0, 1};
    for (int k = 0; k < 16; ++k)
        if (!gfx_finite(v[k])) return "TH019-NONFINITE-MATRIX";
    gfx_set(m, v);
    return 0;
}

/* perspective (:514-530). */
const char* orc_gfx_perspective(float fovy, float aspect, float n, float f, float* m) {
    if (!gfx_finite(fovy) || !gfx_finite(aspect) || !gfx_finite(n) || !gfx_finite(f)) return "TH019-PROJECTION";
    const float pi = 3.14159265358979323846f;
    if (fovy <= 0.0f || fovy >= pi || aspect <= 0.0f || n <= 0.0f || f <= n) return "TH019-PROJECTION";
    const float focal = 1.0f / tanf(fovy * 0.5f);
    const float depthScale = f / (n - f);
    const float fn = f * n;
    const float depthOffset = fn / (n - f);
    const float v[16] = {focal / aspect, 0, 0, 0, 0, focal, 0, 0, 0, 0, depthScale, depthOffset, 0, 0, -1, 0};
    for (int k = 0; k < 16; ++k)
        if (!gfx_finite(v[k])) return "TH019-NONFINITE-MATRIX";
    gfx_set(m, v);
    return 0;
}

/* orthographic (:532-543). */
const char* orc_gfx_orthographic(float l, float r, float b, float t, float n, float f, float* m) {
    if (!gfx_finite(l) || !gfx_finite(r) || !gfx_finite(b) || !gfx_finite(t) || !gfx_finite(n) || !gfx_finite(f))
        return "TH019-PROJECTION";
    if (r <= l || t <= b || n < 0.0f || f <= n) return "TH019-PROJECTION";
    const float v[16] = {2.0f / (r - l), 0, 0, -(r + l) / (r - l),
                         0, 2.0f / (t - b), 0, -(t + b) / (t - b),
                         0, 0, 1.0f / (n - f), n / (n - f),
                         0, 0, 0, 1};
    for (int k = 0; k < 16; ++k)
        if (!gfx_finite(v[k])) return "TH019-NONFINITE-MATRIX";
    gfx_set(m, v);
    return 0;
}

typedef struct {
    float p[4];
    float c[4];
} gfx_clip_vertex;

/* distance to a clip plane (:102-113): Left, Right, Bottom, Top, Near, Far. */
static float gfx_distance(const gfx_clip_vertex* v, int plane) {
    const float* p = v->p;
    switch (plane) {
    case 0: return p[0] + p[3];
    case 1: return p[3] + -p[0];
    case 2: return p[1] + p[3];
    case 3: return p[3] + -p[1];
    case 4: return p[2];
    default: return p[3] + -p[2];
    }
}

static gfx_clip_vertex gfx_interpolate(const gfx_clip_vertex* a, const gfx_clip_vertex* b, float t) {
    gfx_clip_vertex r;
    for (int k = 0; k < 4; ++k) {
        const float dp = b->p[k] + -a->p[k];
        const float sp = t * dp;
        r.p[k] = a->p[k] + sp;
        const float dc = b->c[k] + -a->c[k];
        const float sc = t * dc;
        r.c[k] = a->c[k] + sc;
    }
    return r;
}

/* Sutherland-Hodgman against one plane (:126-149); returns the new count or
 * -1 on TH019-CLIP-NUMERIC. `out` holds at most in + 1 vertices. */
static int gfx_clip_plane(const gfx_clip_vertex* in, int n, int plane, gfx_clip_vertex* out) {
    if (n == 0) return 0;
    int m = 0;
    gfx_clip_vertex prev = in[n - 1];
    float prevDist = gfx_distance(&prev, plane);
    int prevIn = prevDist >= 0.0f;
    for (int i = 0; i < n; ++i) {
        const float dist = gfx_distance(&in[i], plane);
        const int curIn = dist >= 0.0f;
        if (prevIn != curIn) {
            const float den = prevDist + -dist;
            if (den == 0.0f || !gfx_finite(den)) return -1;
            const float amount = prevDist / den;
            if (!gfx_finite(amount)) return -1;
            out[m++] = gfx_interpolate(&prev, &in[i], amount);
        }
        if (curIn) out[m++] = in[i];
        prev = in[i];
        prevDist = dist;
        prevIn = curIn;
    }
    return m;
}

typedef struct {
    double x, y, depth, rw;
    float c[4];
} gfx_screen_vertex;

static double gfx_edge(const gfx_screen_vertex* a, const gfx_screen_vertex* b, double x, double y) {
    const double first = (b->x - a->x) * (y - a->y);
    const double second = (b->y - a->y) * (x - a->x);
    return first - second;
}

static int gfx_top_left(const gfx_screen_vertex* a, const gfx_screen_vertex* b) {
    const double dx = b->x - a->x, dy = b->y - a->y;
    return dy < 0.0 || (dy == 0.0 && dx > 0.0);
}

static int gfx_covered(double v, int inclusive) { return v > 0.0 || (v == 0.0 && inclusive); }

/* prepareScreenTriangle (:348-372). */
static int gfx_screen(const gfx_clip_vertex* t, uint64_t w, uint64_t h, gfx_screen_vertex* s) {
    for (int i = 0; i < 3; ++i) {
        const float cw = t[i].p[3];
        if (!gfx_finite(cw) || cw <= 1.0e-7f) return 0;
        const float x = t[i].p[0] / cw, y = t[i].p[1] / cw, z = t[i].p[2] / cw;
        if (!gfx_finite(x) || !gfx_finite(y) || !gfx_finite(z)) return 0;
        s[i].x = ((double)x * 0.5 + 0.5) * (double)w;
        s[i].y = (0.5 - (double)y * 0.5) * (double)h;
        s[i].depth = z;
        s[i].rw = 1.0 / (double)cw;
        memcpy(s[i].c, t[i].c, sizeof s[i].c);
    }
    const double area = gfx_edge(&s[0], &s[1], s[2].x, s[2].y);
    if (!isfinite(area) || fabs(area) <= 1.0e-12) return 0;
    if (area < 0.0) {
        const gfx_screen_vertex tmp = s[1];
        s[1] = s[2];
        s[2] = tmp;
    }
    return 1;
}

static double gfx_min3(double a, double b, double c) { double m = a < b ? a : b; return m < c ? m : c; }
static double gfx_max3(double a, double b, double c) { double m = a > b ? a : b; return m > c ? m : c; }

/* rasterize (:251-320). */
static void gfx_rasterize(const gfx_screen_vertex* v, uint64_t w, uint64_t h, float* color, float* depth,
                          uint64_t* stats) {
    if (w == 0 || h == 0) return;
    const double area = gfx_edge(&v[0], &v[1], v[2].x, v[2].y);
    int64_t x0 = (int64_t)ceil(gfx_min3(v[0].x, v[1].x, v[2].x) - 0.5);
    int64_t x1 = (int64_t)floor(gfx_max3(v[0].x, v[1].x, v[2].x) - 0.5);
    int64_t y0 = (int64_t)ceil(gfx_min3(v[0].y, v[1].y, v[2].y) - 0.5);
    int64_t y1 = (int64_t)floor(gfx_max3(v[0].y, v[1].y, v[2].y) - 0.5);
    if (x0 < 0) x0 = 0;
    if (y0 < 0) y0 = 0;
    if (x1 > (int64_t)w - 1) x1 = (int64_t)w - 1;
    if (y1 > (int64_t)h - 1) y1 = (int64_t)h - 1;
    if (x0 > x1 || y0 > y1) return;
    const int in0 = gfx_top_left(&v[1], &v[2]), in1 = gfx_top_left(&v[2], &v[0]), in2 = gfx_top_left(&v[0], &v[1]);
    for (int64_t y = y0; y <= y1; ++y)
        for (int64_t x = x0; x <= x1; ++x) {
            const double cx = (double)x + 0.5, cy = (double)y + 0.5;
            const double e0 = gfx_edge(&v[1], &v[2], cx, cy);
            const double e1 = gfx_edge(&v[2], &v[0], cx, cy);
            const double e2 = gfx_edge(&v[0], &v[1], cx, cy);
            if (!gfx_covered(e0, in0) || !gfx_covered(e1, in1) || !gfx_covered(e2, in2)) continue;
            const double w0 = e0 / area, w1 = e1 / area, w2 = e2 / area;
            double d = w0 * v[0].depth + w1 * v[1].depth + w2 * v[2].depth;
            if (!isfinite(d) || d < -1.0e-6 || d > 1.0 + 1.0e-6) continue;
            d = d < 0.0 ? 0.0 : (d > 1.0 ? 1.0 : d);
            const double den = w0 * v[0].rw + w1 * v[1].rw + w2 * v[2].rw;
            if (!isfinite(den) || den <= 0.0) continue;
            float c[4];
            int valid = 1;
            for (int k = 0; k < 4; ++k) {
                const double num = w0 * (double)v[0].c[k] * v[0].rw + w1 * (double)v[1].c[k] * v[1].rw +
                                   w2 * (double)v[2].c[k] * v[2].rw;
                const double value = num / den;
                if (!isfinite(value)) { valid = 0; break; }
                c[k] = (float)(value < 0.0 ? 0.0 : (value > 1.0 ? 1.0 : value));
            }
            if (!valid) continue;
            ++stats[2];
            const uint64_t pixel = (uint64_t)y * w + (uint64_t)x;
            if (!((float)d < depth[pixel])) continue;
            depth[pixel] = (float)d;
            memcpy(&color[pixel * 4], c, sizeof c);
            ++stats[3];
        }
}

/* render (:574-596) with prepareRender (:374-421). */
const char* orc_render(const float* positions, uint64_t vertices, const int64_t* indices, uint64_t triangles,
                       const float* colors, const float* model, const float* view, const float* projection,
                       uint64_t width, uint64_t height, const float* clear, float* color, float* depth,
                       uint64_t* stats) {
    for (uint64_t k = 0; k < vertices * 3; ++k)
        if (!gfx_finite(positions[k])) return "TH019-NONFINITE-VERTEX";
    for (uint64_t k = 0; k < vertices * 4; ++k)
        if (!gfx_finite(colors[k]) || colors[k] < 0.0f || colors[k] > 1.0f) return "TH019-COLOR-RANGE";
    for (uint64_t k = 0; k < triangles * 3; ++k)
        if (indices[k] < 0 || (uint64_t)indices[k] >= vertices) return "TH019-INDEX";
    for (int k = 0; k < 4; ++k)
        if (!gfx_finite(clear[k]) || clear[k] < 0.0f || clear[k] > 1.0f) return "TH019-CLEAR-COLOR";
    for (int k = 0; k < 16; ++k)
        if (!gfx_finite(model[k]) || !gfx_finite(view[k]) || !gfx_finite(projection[k])) return "TH019-NONFINITE-MATRIX";
    float mv[16], mvp[16];
    orc_gfx_multiply(view, model, mv);
    orc_gfx_multiply(projection, mv, mvp);
    gfx_clip_vertex* clip = (gfx_clip_vertex*)malloc(sizeof(gfx_clip_vertex) * (vertices ? vertices : 1));
    for (uint64_t v = 0; v < vertices; ++v) {
        const float in[4] = {positions[v * 3], positions[v * 3 + 1], positions[v * 3 + 2], 1.0f};
        for (int row = 0; row < 4; ++row) {
            float acc = 0.0f;
            for (int col = 0; col < 4; ++col) {
                const float p = mvp[row * 4 + col] * in[col];
                acc = acc + p;
            }
            if (!gfx_finite(acc)) { free(clip); return "TH019-NONFINITE-TRANSFORMED"; }
            clip[v].p[row] = acc;
        }
        memcpy(clip[v].c, &colors[v * 4], 4 * sizeof(float));
    }
    const uint64_t pixels = width * height;
    for (uint64_t p = 0; p < pixels; ++p) {
        memcpy(&color[p * 4], clear, 4 * sizeof(float));
        depth[p] = INFINITY;
    }
    stats[0] = triangles;
    stats[1] = stats[2] = stats[3] = 0;
    gfx_clip_vertex poly[2][16];
    for (uint64_t t = 0; t < triangles; ++t) {
        int n = 3;
        for (int c = 0; c < 3; ++c) poly[0][c] = clip[indices[t * 3 + c]];
        int cur = 0;
        for (int plane = 0; plane < 6 && n >= 3; ++plane) {
            n = gfx_clip_plane(poly[cur], n, plane, poly[cur ^ 1]);
            if (n < 0) { free(clip); return "TH019-CLIP-NUMERIC"; }
            cur ^= 1;
        }
        if (n < 3) continue;
        for (int c = 1; c + 1 < n; ++c) {
            ++stats[1];
            const gfx_clip_vertex tri[3] = {poly[cur][0], poly[cur][c], poly[cur][c + 1]};
            gfx_screen_vertex s[3];
            if (gfx_screen(tri, width, height, s)) gfx_rasterize(s, width, height, color, depth, stats);
        }
    }
    free(clip);
    return 0;
}
