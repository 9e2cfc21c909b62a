// Fused CSTAdamW step: AdamW moments and proposal, field_lrs rescale and the
// coordinate law, one thread per atom row with 16-byte loads and stores.
//
// Arithmetic is written as separate round-to-nearest float32 operations in the
// order torch's single-tensor AdamW and torchcst's coordinate updates use
// (optim/adamw.py:249-294 -> torch.optim.adam._single_tensor_adam;
// optim/_field_lrs.py:128-134; _backends/torch/updates/rational_radius.py:10-29;
// _backends/torch/algorithms/polar_update/executor.py:42-112 and :168-176), so
// results match the CPU oracle bit for bit. The exp_avg lerp uses a fused
// multiply-add like torch's vectorized CPU lerp.

#include "common.cuh"

namespace tcst {

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

__device__ __forceinline__ float adam_one(float p, float g, float &m, float &v,
                                          const tcst_adamw &h) {
    if (h.has_decay) p = fmul(p, h.decay_factor);
    m = __fmaf_rn(h.lerp_weight, fsub(g, m), m);
    v = fadd(fmul(v, h.beta2), fmul(fmul(h.one_minus_beta2, g), g));
    float denom = fadd(fdiv(fsqrt(v), h.bias2_sqrt), h.eps);
    return fadd(p, fdiv(fmul(h.neg_step_size, m), denom));
}

__device__ __forceinline__ float field(float point, float prev, int c, const tcst_adamw &h) {
    if (!(h.field_mask >> c & 1)) return point;
    return fadd(prev, fmul(fsub(point, prev), h.field_ratio[c]));
}

__device__ __forceinline__ float torus(float x, float period) {
    // torch.remainder for floating point: fmod, then shift to the divisor's sign.
    float mod = fmodf(x, period);
    if (mod != 0.0f && ((mod < 0.0f) != (period < 0.0f))) mod = fadd(mod, period);
    return mod;
}

__device__ __forceinline__ float4 coordinate_law(float4 prev, float4 pt, int kind,
                                                 const tcst_adamw &h) {
    // displacement = proposal - previous; the coordinate law restarts from previous.
    float4 d = make_float4(fsub(pt.x, prev.x), fsub(pt.y, prev.y), fsub(pt.z, prev.z),
                           fsub(pt.w, prev.w));
    float4 out;
    if (kind == TCST_RATIONAL) {
        const float cap = h.amplitude_cap;
        out.x = fminf(fmaxf(fadd(prev.x, d.x), -cap), cap);
        out.y = fminf(fmaxf(fadd(prev.y, d.y), 0.0f), 1.0f);
        out.z = fadd(prev.z, d.z);
        out.w = fadd(prev.w, d.w);
    } else {
        // _project_polar (executor.py:168-176).
        const float tiny = 1.17549435e-38f;
        float rs = fadd(fmul(prev.x, prev.x), fmul(prev.y, prev.y));
        float safe_r = fsqrt(fmaxf(rs, tiny));
        float ux = 0.0f, uy = 1.0f;
        if (rs > tiny) {
            ux = fdiv(prev.x, safe_r);
            uy = fdiv(prev.y, safe_r);
        }
        float rad = fminf(fmaxf(safe_r, 1.0f), 2.0f);
        float px = fmul(ux, rad), py = fmul(uy, rad);
        // Tangential task motion and activity (executor.py:59-98).
        float radius_square = fadd(fmul(px, px), fmul(py, py));
        float dot = fadd(fmul(d.x, px), fmul(d.y, py));
        float radial = fdiv(dot, radius_square);
        float tx = fsub(d.x, fmul(radial, px)), ty = fsub(d.y, fmul(radial, py));
        float cx = fadd(px, tx), cy = fadd(py, ty);
        float chord_q = fadd(fmul(cx, cx), fmul(cy, cy));
        float cs = fsqrt(chord_q);
        float dx = fdiv(cx, cs), dy = fdiv(cy, cs);
        float energy = fadd(fmul(tx, tx), fmul(ty, ty));
        if (h.polar_energy_step != 0.0f) energy = fdiv(energy, h.polar_energy_step);
        float drs = fadd(fmul(dx, dx), fmul(dy, dy));
        float amp = fdiv(fmul(h.polar_amplitude_max, dx), fsqrt(fmaxf(drs, tiny)));
        float ratio = fdiv(amp, h.polar_w_c);
        float dormant = fdiv(1.0f, fadd(1.0f, fmul(ratio, ratio)));
        float dormant_q = fmul(h.polar_dormant_q_scale, dormant);
        float task_q = fadd(radius_square, fmul(h.polar_activity_gain, energy));
        task_q = fminf(fmaxf(fadd(task_q, dormant_q), 1.0f), 4.0f);
        float sq = fsqrt(task_q);
        float tpx = fmul(dx, sq), tpy = fmul(dy, sq);
        float activity = fdiv(fsub(task_q, 1.0f), task_q);
        float reg_q = fdiv(1.0f, fsub(1.0f, fmul(activity, h.polar_decay)));
        float scale = fsqrt(fdiv(reg_q, task_q));
        out.x = fmul(tpx, scale);
        out.y = fmul(tpy, scale);
        // Flat-torus retraction of both centers (flat_torus.py:30-35).
        out.z = torus(fadd(prev.z, d.z), h.period_out);
        out.w = torus(fadd(prev.w, d.w), h.period_in);
        if (h.amplitude_decay != 0.0f) {
            // decay_amplitude (executor.py:18-41): subtract the decayed old
            // normalized amplitude at the accepted radius, keep t's sign.
            float old_r = fsqrt(fmaxf(fadd(fmul(prev.x, prev.x), fmul(prev.y, prev.y)), tiny));
            float new_r = fsqrt(fmaxf(fadd(fmul(out.x, out.x), fmul(out.y, out.y)), tiny));
            float old_amp = fdiv(prev.x, old_r);
            float target = fsub(fdiv(out.x, new_r), fmul(h.amplitude_decay, old_amp));
            target = fminf(fmaxf(target, -1.0f), 1.0f);
            float absolute = fabsf(target);
            float room = fmaxf(fmul(fsub(1.0f, absolute), fadd(1.0f, absolute)), 0.0f);
            float magnitude = fmul(new_r, fsqrt(room));
            out.x = fmul(new_r, target);
            out.y = copysignf(magnitude, out.y);
        }
    }
    return out;
}

__device__ __forceinline__ void step_row(long long a, float4 *__restrict__ p,
                                         const float4 *__restrict__ grad, float4 *__restrict__ m,
                                         float4 *__restrict__ v, int kind, const tcst_adamw &h) {
    float4 prev = p[a], g = grad[a], mm = m[a], vv = v[a];
    float4 pt;
    pt.x = adam_one(prev.x, g.x, mm.x, vv.x, h);
    pt.y = adam_one(prev.y, g.y, mm.y, vv.y, h);
    pt.z = adam_one(prev.z, g.z, mm.z, vv.z, h);
    pt.w = adam_one(prev.w, g.w, mm.w, vv.w, h);
    m[a] = mm;
    v[a] = vv;
    pt.x = field(pt.x, prev.x, 0, h);
    pt.y = field(pt.y, prev.y, 1, h);
    pt.z = field(pt.z, prev.z, 2, h);
    pt.w = field(pt.w, prev.w, 3, h);
    p[a] = coordinate_law(prev, pt, kind, h);
}

__global__ void optimizer_kernel(float4 *__restrict__ p, const float4 *__restrict__ grad,
                                 float4 *__restrict__ m, float4 *__restrict__ v,
                                 long long atoms, int kind, tcst_adamw h) {
    pdl_wait();
    const long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (a < atoms) step_row(a, p, grad, m, v, kind, h);
}

// Same step with the scalars read from device memory when the kernel runs.
__global__ void optimizer_dev_kernel(float4 *__restrict__ p, const float4 *__restrict__ grad,
                                     float4 *__restrict__ m, float4 *__restrict__ v,
                                     long long atoms, int kind,
                                     const tcst_adamw *__restrict__ hp) {
    pdl_wait();
    __shared__ tcst_adamw h;
    if (threadIdx.x == 0) h = *hp;
    __syncthreads();
    const long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (a < atoms) step_row(a, p, grad, m, v, kind, h);
}

// Scalar ring: one CTA copies the slot of use count c from the host ring
// (device mapping, ld.global.cv so that no cached copy of an earlier use of
// the slot is seen; one 16-byte load per thread, all in flight together) into
// the device state block [count, valid, -, -, tcst_adamw]. Nothing here
// depends on the preceding kernels (the state is written only by earlier
// fetches, which have completed), so it runs before the dependency wait.
__global__ void scalar_ring_fetch_kernel(const uint4 *ring, int slots, long long slot_vecs,
                                         unsigned *state, unsigned *status) {
    constexpr int VECS = int(TCST_RING_SEQ_OFFSET / 16);
    __shared__ uint4 buf[VECS + 1];
    const unsigned c = state[0];
    const uint4 *slot = ring + (long long)(c % unsigned(slots)) * slot_vecs;
    if (threadIdx.x <= VECS) {
        uint4 v;
        asm volatile("ld.global.cv.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(slot + threadIdx.x));
        buf[threadIdx.x] = v;
    }
    __syncthreads();
    pdl_wait();
    const bool ok = buf[VECS].x == c;
    if (threadIdx.x < VECS) reinterpret_cast<uint4 *>(state + 4)[threadIdx.x] = buf[threadIdx.x];
    if (threadIdx.x == 0) {
        state[1] = ok ? 1u : 0u;
        state[0] = c + 1u;
        if (!ok) atomicOr(status, TCST_STATUS_SEQUENCE);
    }
}

// The optimizer step with the scalars of a fetched ring state block.
__global__ void optimizer_ring_kernel(float4 *__restrict__ p, const float4 *__restrict__ grad,
                                      float4 *__restrict__ m, float4 *__restrict__ v,
                                      long long atoms, int kind, const unsigned *__restrict__ state) {
    pdl_wait();
    __shared__ tcst_adamw h;
    __shared__ bool ok;
    if (threadIdx.x == 0) {
        ok = state[1] != 0u;
        h = *reinterpret_cast<const tcst_adamw *>(state + 4);
    }
    __syncthreads();
    const long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (ok && a < atoms) step_row(a, p, grad, m, v, kind, h);
}

// The coordinate law alone: proposal (written by an outside AdamW and field
// rescale) is replaced in place by the law applied from previous.
__global__ void coordinate_update_kernel(float4 *__restrict__ proposal,
                                         const float4 *__restrict__ previous, long long atoms,
                                         int kind, tcst_adamw h) {
    pdl_wait();
    const long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (a < atoms) proposal[a] = coordinate_law(previous[a], proposal[a], kind, h);
}

} // namespace tcst

using namespace tcst;

extern "C" int tcst_optimizer_step(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                                   float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                                   const tcst_adamw *params, void *stream) {
    if (atoms < 0 || !params || (kind != TCST_RATIONAL && kind != TCST_POLAR) ||
        (atoms && (!p_dev || !grad_dev || !exp_avg_dev || !exp_avg_sq_dev))) {
        tcst_set_error("tcst_optimizer_step: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(p_dev) | reinterpret_cast<uintptr_t>(grad_dev) |
         reinterpret_cast<uintptr_t>(exp_avg_dev) | reinterpret_cast<uintptr_t>(exp_avg_sq_dev)) %
        16) {
        tcst_set_error("tcst_optimizer_step: tensors must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (kind == TCST_RATIONAL && params->amplitude_decay != 0.0f) {
        tcst_set_error("tcst_optimizer_step: amplitude decay requires Polar atoms");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    TCST_CUDA(launch_pdl(optimizer_kernel, dim3(unsigned((atoms + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, 
        (float4 *)p_dev, (const float4 *)grad_dev, (float4 *)exp_avg_dev, (float4 *)exp_avg_sq_dev,
        atoms, kind, *params));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_optimizer_step_device(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                                          float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                                          const tcst_adamw *params_dev, void *stream) {
    if (atoms < 0 || !params_dev || (kind != TCST_RATIONAL && kind != TCST_POLAR) ||
        (atoms && (!p_dev || !grad_dev || !exp_avg_dev || !exp_avg_sq_dev))) {
        tcst_set_error("tcst_optimizer_step_device: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(p_dev) | reinterpret_cast<uintptr_t>(grad_dev) |
         reinterpret_cast<uintptr_t>(exp_avg_dev) | reinterpret_cast<uintptr_t>(exp_avg_sq_dev) |
         reinterpret_cast<uintptr_t>(params_dev)) %
        16) {
        tcst_set_error("tcst_optimizer_step_device: pointers must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    TCST_CUDA(launch_pdl(optimizer_dev_kernel, dim3(unsigned((atoms + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, 
        (float4 *)p_dev, (const float4 *)grad_dev, (float4 *)exp_avg_dev, (float4 *)exp_avg_sq_dev,
        atoms, kind, params_dev));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_scalar_ring_fetch(const void *ring_host, int32_t slots, int64_t slot_bytes,
                                      void *ring_state_dev, uint32_t *status_dev, void *stream) {
    if (!ring_host || slots < 1 || slot_bytes < (int64_t)TCST_RING_SLOT_MIN || slot_bytes % 16 ||
        !ring_state_dev || !status_dev) {
        tcst_set_error("tcst_scalar_ring_fetch: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(ring_host) | reinterpret_cast<uintptr_t>(ring_state_dev)) %
        16) {
        tcst_set_error("tcst_scalar_ring_fetch: the ring and the state block must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    // The kernel reads the ring through its device mapping.
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ring_host) != cudaSuccess ||
        attr.type != cudaMemoryTypeHost || !attr.devicePointer) {
        cudaGetLastError();
        tcst_set_error("tcst_scalar_ring_fetch: the ring must be pinned, device-mapped host memory");
        return TCST_ERR_ARGUMENT;
    }
    TCST_CUDA(launch_pdl(scalar_ring_fetch_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream,
                         static_cast<const uint4 *>(attr.devicePointer), int(slots),
                         (long long)(slot_bytes / 16), static_cast<unsigned *>(ring_state_dev),
                         status_dev));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_optimizer_step_ring(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                                        float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                                        const void *ring_state_dev, void *stream) {
    if (atoms < 0 || !ring_state_dev || (kind != TCST_RATIONAL && kind != TCST_POLAR) ||
        (atoms && (!p_dev || !grad_dev || !exp_avg_dev || !exp_avg_sq_dev))) {
        tcst_set_error("tcst_optimizer_step_ring: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(p_dev) | reinterpret_cast<uintptr_t>(grad_dev) |
         reinterpret_cast<uintptr_t>(exp_avg_dev) | reinterpret_cast<uintptr_t>(exp_avg_sq_dev) |
         reinterpret_cast<uintptr_t>(ring_state_dev)) %
        16) {
        tcst_set_error("tcst_optimizer_step_ring: pointers must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    TCST_CUDA(launch_pdl(optimizer_ring_kernel, dim3(unsigned((atoms + 255) / 256)), dim3(256), 0,
                         (cudaStream_t)stream, (float4 *)p_dev, (const float4 *)grad_dev,
                         (float4 *)exp_avg_dev, (float4 *)exp_avg_sq_dev, atoms, kind,
                         static_cast<const unsigned *>(ring_state_dev)));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_coordinate_update(float *proposal_dev, const float *previous_dev,
                                      int64_t atoms, int32_t kind, const tcst_adamw *params,
                                      void *stream) {
    if (atoms < 0 || !params || (kind != TCST_RATIONAL && kind != TCST_POLAR) ||
        (atoms && (!proposal_dev || !previous_dev))) {
        tcst_set_error("tcst_coordinate_update: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(proposal_dev) | reinterpret_cast<uintptr_t>(previous_dev)) %
        16) {
        tcst_set_error("tcst_coordinate_update: tensors must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (proposal_dev == previous_dev && atoms) {
        tcst_set_error("tcst_coordinate_update: previous must not alias the proposal");
        return TCST_ERR_ARGUMENT;
    }
    if (kind == TCST_RATIONAL && params->amplitude_decay != 0.0f) {
        tcst_set_error("tcst_coordinate_update: amplitude decay requires Polar atoms");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    TCST_CUDA(launch_pdl(coordinate_update_kernel, dim3(unsigned((atoms + 255) / 256)), dim3(256),
                         0, (cudaStream_t)stream, (float4 *)proposal_dev,
                         (const float4 *)previous_dev, atoms, kind, *params));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
