// The optimizer's per-parameter update, shared by the standalone SGD pass
// (mlp.cu) and the weight-gradient GEMM epilogue that applies it in place
// (gemm.cu), so both produce the same bits.
#pragma once

namespace thb {

// One parameter update (src/training/v0/Training.cpp:366-372): d = g, or with
// momentum d = v*mu + g and v = d; p = p - d*lr. Each operation rounds to f32
// (no contraction into FMAs).
__device__ __forceinline__ float sgdStep(float p, float g, float* v, float lr, float mu) {
    float d = g;
    if (v) {
        d = __fadd_rn(__fmul_rn(*v, mu), g);
        *v = d;
    }
    return __fsub_rn(p, __fmul_rn(d, lr));
}

} // namespace thb
