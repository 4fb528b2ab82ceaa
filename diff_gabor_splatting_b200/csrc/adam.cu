// Fused Adam step over the parameter tensors of a scene batch.
//
// The reference's optimisation loop (examples/fit_texture.py:50-61) calls
// torch.optim.Adam after every render backward; its default multi-tensor path issues
// about ten element-wise passes over the parameters, moments and gradients per step
// (torch/optim/adam.py, _multi_tensor_adam).  Here one launch updates every tensor:
// each element is read once (parameter, gradient, both moments: 16 bytes) and written
// once (parameter, moments: 12 bytes), HBM-bound at 28 bytes per element.
//
// The arithmetic follows torch's order per element (weight decay added to the
// gradient, m = lerp(m, g, 1 - beta1), v = v * beta2 + (1 - beta2) g g, then
// p += -(lr / bias_correction1) * m / (sqrt(v) / sqrt(bias_correction2) + eps)), with
// the bias corrections computed in double on the host as torch does.
//
// The capturable form (gs_adam_step_capturable) keeps each tensor's step count on the
// device, as torch.optim.Adam(capturable=True) does: one small launch increments the
// counts, and the update computes the bias corrections from them (in double), so the
// step can be recorded in a CUDA graph and replayed with the count advancing.  An
// optional device flag lets a recorded step skip itself (counts and update) when the
// step that produced the gradients went wrong -- for a graphed training step, when the
// render's binning overflowed its arena and rendered background only.
#include "common.cuh"

namespace gs {
namespace {

constexpr int kAdamTensors = 48;          // tensors per launch (kernel-parameter table)
constexpr int kAdamThreads = 256;
constexpr int kAdamChunk = kAdamThreads * 4 * 8;   // elements per block: 8 float4 per thread

struct AdamTable {
    float* param[kAdamTensors];
    const float* grad[kAdamTensors];
    float* exp_avg[kAdamTensors];
    float* exp_avg_sq[kAdamTensors];
    int64_t size[kAdamTensors];
    int64_t first_block[kAdamTensors + 1];   // block range of each tensor
    int tensors;
    bool vector[kAdamTensors];                // all four arrays 16-byte aligned
    float beta1_weight, beta2, beta2_weight, eps, weight_decay, step_size, bias2_sqrt;
    // capturable form: per-tensor step counts on the device (NULL: host scalars above)
    const float* step[kAdamTensors];
    double lr, beta1_d, beta2_d;
    // capturable form: device flag (NULL: none); nonzero skips the whole step
    const int32_t* skip;
};

struct AdamScalars {
    float beta1_weight, beta2, beta2_weight, eps, weight_decay, step_size, bias2_sqrt;
};

__device__ __forceinline__ void adam_element(float& p, float g, float& m, float& v,
                                             const AdamScalars& s) {
    if (s.weight_decay != 0.f) g = fmaf(s.weight_decay, p, g);
    m = fmaf(s.beta1_weight, g - m, m);                 // lerp(m, g, 1 - beta1), weight < 0.5
    v = v * s.beta2;
    v = fmaf(s.beta2_weight * g, g, v);                 // addcmul(v, g, g, 1 - beta2)
    const float denom = sqrtf(v) / s.bias2_sqrt + s.eps;
    p = fmaf(s.step_size, m / denom, p);                // addcdiv(p, m, denom, -lr / bc1)
}

__global__ __launch_bounds__(kAdamThreads) void adam_kernel(const AdamTable T) {
    AdamScalars s{T.beta1_weight, T.beta2, T.beta2_weight, T.eps, T.weight_decay,
                  T.step_size, T.bias2_sqrt};
    if (T.skip && *T.skip) return;   // e.g. the render's binning overflowed its arena
    const int64_t block = blockIdx.x;
    int t = 0;
    while (t + 1 < T.tensors && T.first_block[t + 1] <= block) ++t;   // <= 48 tensors
    if (T.step[t]) {   // bias corrections of this tensor's device step count, in double
        const double step = double(*T.step[t]);
        s.step_size = float(-(T.lr / (1.0 - pow(T.beta1_d, step))));
        s.bias2_sqrt = float(sqrt(1.0 - pow(T.beta2_d, step)));
    }
    const int64_t begin = (block - T.first_block[t]) * kAdamChunk;
    const int64_t end = min(begin + kAdamChunk, T.size[t]);
    float* __restrict__ param = T.param[t];
    const float* __restrict__ grad = T.grad[t];
    float* __restrict__ m1 = T.exp_avg[t];
    float* __restrict__ m2 = T.exp_avg_sq[t];
    if (T.vector[t]) {
        const int64_t vec_end = begin + ((end - begin) & ~int64_t(3));
        for (int64_t i = begin + 4 * threadIdx.x; i < vec_end; i += 4 * kAdamThreads) {
            float4 p = *reinterpret_cast<const float4*>(param + i);
            const float4 g = __ldg(reinterpret_cast<const float4*>(grad + i));
            float4 m = *reinterpret_cast<const float4*>(m1 + i);
            float4 v = *reinterpret_cast<const float4*>(m2 + i);
            adam_element(p.x, g.x, m.x, v.x, s);
            adam_element(p.y, g.y, m.y, v.y, s);
            adam_element(p.z, g.z, m.z, v.z, s);
            adam_element(p.w, g.w, m.w, v.w, s);
            *reinterpret_cast<float4*>(param + i) = p;
            *reinterpret_cast<float4*>(m1 + i) = m;
            *reinterpret_cast<float4*>(m2 + i) = v;
        }
        for (int64_t i = vec_end + threadIdx.x; i < end; i += kAdamThreads)
            adam_element(param[i], grad[i], m1[i], m2[i], s);
    } else {
        for (int64_t i = begin + threadIdx.x; i < end; i += kAdamThreads)
            adam_element(param[i], grad[i], m1[i], m2[i], s);
    }
}

// Advance each tensor's device step count by one (before the update reads it).
__global__ void adam_count_kernel(AdamTable T) {
    if (T.skip && *T.skip) return;
    const int t = threadIdx.x;
    if (t < T.tensors) *const_cast<float*>(T.step[t]) += 1.f;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Shared by both entry points: tables of up to kAdamTensors non-empty tensors, one
// update launch each (preceded, with device step counts, by the count launch).
int adam_launches(const char* fn, int tensors, float* const* params, const float* const* grads,
                  float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* sizes,
                  float* const* steps, const int32_t* skip, double lr, double beta1,
                  double beta2, double eps, double weight_decay, double bias1, double bias2,
                  cudaStream_t s) {
    if (tensors < 0 || (tensors > 0 && (!params || !grads || !exp_avgs || !exp_avg_sqs || !sizes)))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid tensor table");
    if (!(lr >= 0.0) || !(eps >= 0.0) || !(beta1 >= 0.0 && beta1 < 1.0) ||
        !(beta2 >= 0.0 && beta2 < 1.0) || !(weight_decay >= 0.0))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid hyper-parameters");
    for (int t = 0; t < tensors; ++t) {
        if (sizes[t] < 0) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": negative tensor size");
        if (sizes[t] > 0 && (!params[t] || !grads[t] || !exp_avgs[t] || !exp_avg_sqs[t] ||
                             (steps && !steps[t])))
            return fail(GS_ERR_ARGUMENT, std::string(fn) + ": NULL tensor");
    }
    for (int first = 0; first < tensors; first += kAdamTensors) {
        AdamTable T{};
        T.tensors = 0;
        int64_t blocks = 0;
        for (int t = first; t < tensors && t < first + kAdamTensors; ++t) {
            if (sizes[t] == 0) continue;
            const int k = T.tensors++;
            T.param[k] = params[t];
            T.grad[k] = grads[t];
            T.exp_avg[k] = exp_avgs[t];
            T.exp_avg_sq[k] = exp_avg_sqs[t];
            T.size[k] = sizes[t];
            T.step[k] = steps ? steps[t] : nullptr;
            T.vector[k] = aligned16(params[t]) && aligned16(grads[t]) && aligned16(exp_avgs[t]) &&
                          aligned16(exp_avg_sqs[t]);
            T.first_block[k] = blocks;
            blocks += (sizes[t] + kAdamChunk - 1) / kAdamChunk;
        }
        if (T.tensors == 0) continue;
        T.first_block[T.tensors] = blocks;
        if (blocks > INT_MAX) return fail(GS_ERR_LIMIT, std::string(fn) + ": tensors too large");
        T.beta1_weight = float(1.0 - beta1);
        T.beta2 = float(beta2);
        T.beta2_weight = float(1.0 - beta2);
        T.eps = float(eps);
        T.weight_decay = float(weight_decay);
        T.step_size = float(-(lr / bias1));
        T.bias2_sqrt = float(std::sqrt(bias2));
        T.lr = lr;
        T.beta1_d = beta1;
        T.beta2_d = beta2;
        T.skip = skip;
        if (steps) {
            adam_count_kernel<<<1, kAdamTensors, 0, s>>>(T);
            GS_CHECK_LAUNCH("adam_count_kernel");
        }
        adam_kernel<<<unsigned(blocks), kAdamThreads, 0, s>>>(T);
        GS_CHECK_LAUNCH("adam_kernel");
    }
    return GS_OK;
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" int gs_adam_step(int tensors, float* const* params, const float* const* grads,
                            float* const* exp_avgs, float* const* exp_avg_sqs,
                            const int64_t* sizes, double lr, double beta1, double beta2,
                            double eps, double weight_decay, int64_t step, void* stream) {
    if (step < 1) return fail(GS_ERR_ARGUMENT, "gs_adam_step: step counts from 1");
    // bias corrections in double, as torch.optim.Adam computes them in Python
    const double bias1 = 1.0 - std::pow(beta1, double(step));
    const double bias2 = 1.0 - std::pow(beta2, double(step));
    return adam_launches("gs_adam_step", tensors, params, grads, exp_avgs, exp_avg_sqs, sizes,
                         nullptr, nullptr, lr, beta1, beta2, eps, weight_decay, bias1, bias2,
                         as_stream(stream));
}

extern "C" int gs_adam_step_capturable(int tensors, float* const* params,
                                       const float* const* grads, float* const* exp_avgs,
                                       float* const* exp_avg_sqs, const int64_t* sizes,
                                       float* const* steps, double lr, double beta1,
                                       double beta2, double eps, double weight_decay,
                                       const int32_t* skip, void* stream) {
    if (tensors > 0 && !steps)
        return fail(GS_ERR_ARGUMENT, "gs_adam_step_capturable: NULL step table");
    return adam_launches("gs_adam_step_capturable", tensors, params, grads, exp_avgs,
                         exp_avg_sqs, sizes, steps, skip, lr, beta1, beta2, eps, weight_decay,
                         1.0, 1.0, as_stream(stream));
}
