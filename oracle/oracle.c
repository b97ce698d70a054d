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
            /* Evaluator.cpp:125-154: sequential-k f32, each op rounded */
            const value_t* d1 = &vals[position_of(r, n->dependencies[1])];
            v->shape[0] = d0->shape[0];
            v->shape[1] = d1->shape[1];
            v->count = v->shape[0] * v->shape[1];
            v->data = malloc(4 * (v->count ? v->count : 1));
            v->owned = 1;
            orc_matmul_f32((const float*)d0->data, (const float*)d1->data, (float*)v->data, d0->shape[0], d0->shape[1],
                           d1->shape[1]);
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
        case THB_OP_SOFTMAX: case THB_OP_ROW_MAX: case THB_OP_SUM: {
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
