// Scalar steps of the hyper-connection mixer shared by its kernels (hc.cu) and the persistent
// mixer + shared-expert decode (f3stack.cu), in the reference's two rounding regimes
// (mlx-qwen38/cpp/src/kernels.cpp:1363-1560: fused decode kernels for <= 16 rows, the prefill
// path's per-op bf16 roundings above).
#pragma once

#include "common.cuh"
#include "qlinear.cuh"

namespace moe_qlin {

constexpr int kHcStreams = 4;                    // hc_count of the reference's models

// mix = silu(d / HC) in the row count's regime
MOE_D float hc_mix_value(float d, int prefill) {
    if (prefill) {
        const float v = bf16r(__fdiv_rn(bf16r(d), (float)kHcStreams));
        return __fmul_rn(v, sigmoid_bf16(v));
    }
    const float v = __fdiv_rn(d, (float)kHcStreams);
    return __fmul_rn(v, sigmoidf(v));
}

// inj = 2 * sigmoid(iv / HC) in the row count's regime
MOE_D float hc_inj_value(float iv, int prefill) {
    if (prefill) return __fmul_rn(2.0f, sigmoid_bf16(bf16r(__fdiv_rn(bf16r(iv), (float)kHcStreams))));
    return __fmul_rn(2.0f, sigmoidf(__fdiv_rn(iv, (float)kHcStreams)));
}

}  // namespace moe_qlin
