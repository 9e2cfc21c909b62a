// Dense weight assembly W = sum_a amp_a m_out,a (x) m_in,a, and the TF32 split.
//
// Each warp owns one atom: lanes evaluate the input-axis masses of a 32-column
// strip, output-axis masses are broadcast row by row with shuffles, and every
// product is added into a 64-bit fixed-point accumulator (2^-40 units) with a
// reduction that is exact, hence independent of the order in which atoms land.
// The finalize pass converts to float32, writes the two-term TF32 split planes
// that the tensor-core GEMMs consume, and clears the accumulator for the next
// call.

#include "common.cuh"

namespace tcst {

constexpr float FIXED_SCALE = 1099511627776.0f; // 2^40
constexpr double FIXED_UNIT = 1.0 / 1099511627776.0;

__device__ __forceinline__ void red_add_u64(unsigned long long *addr, long long v) {
    asm volatile("red.global.add.u64 [%0], %1;" ::"l"(addr), "l"((unsigned long long)v)
                 : "memory");
}

__device__ __forceinline__ float tf32_rna(float x) {
    unsigned r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__global__ void __launch_bounds__(256) weight_scatter_kernel(
    const float *__restrict__ table, int words, long long atoms, AxisCfg out_ax, AxisCfg in_ax,
    unsigned long long *__restrict__ acc) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (gridDim.x * (long long)blockDim.x) >> 5;
    const int aw = axis_words(out_ax.modes);
    const int ni = in_ax.sites, no = out_ax.sites;
    for (long long a = warp; a < atoms; a += nwarps) {
        const float *rec = table + a * (long long)words;
        const float *ob = rec + 4;
        const float *ib = rec + 4 + aw;
        const int fo = reinterpret_cast<const int *>(ob)[1];
        const int fi = reinterpret_cast<const int *>(ib)[1];
        if (fo == 0 || fi == 0) continue;
        const int first_o = reinterpret_cast<const int *>(ob)[0];
        const int first_i = reinterpret_cast<const int *>(ib)[0];
        const float amp = rec[0];
        for (int r0 = 0; r0 < fo; r0 += 32) {
            const int rows = min(32, fo - r0);
            float mo = (lane < rows) ? amp * site_mass(ob, out_ax.modes, r0 + lane, fo) : 0.0f;
            int orow = wrap_site((long long)first_o + r0 + lane, no);
            for (int c0 = 0; c0 < fi; c0 += 32) {
                const int c = c0 + lane;
                const bool cv = c < fi;
                const float mi = cv ? site_mass(ib, in_ax.modes, c, fi) * FIXED_SCALE : 0.0f;
                const int col = wrap_site((long long)first_i + c, ni);
                for (int rr = 0; rr < rows; ++rr) {
                    const float v = __shfl_sync(0xffffffffu, mo, rr) * mi;
                    const int row = __shfl_sync(0xffffffffu, orow, rr);
                    if (cv) red_add_u64(acc + (long long)row * ni + col, __float2ll_rn(v));
                }
            }
        }
    }
}

__global__ void weight_finalize_kernel(unsigned long long *__restrict__ acc, int no, int ni,
                                       float *__restrict__ w, long long ldw,
                                       float *__restrict__ hi, float *__restrict__ lo,
                                       long long lds) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long total = (long long)no * ni;
    if (idx >= total) return;
    int o = int(idx / ni), i = int(idx % ni);
    long long fixed = (long long)acc[idx];
    acc[idx] = 0ull;
    float v = float(double(fixed) * FIXED_UNIT);
    if (w) w[o * ldw + i] = v;
    if (hi) {
        float h = tf32_rna(v);
        hi[o * lds + i] = h;
        lo[o * lds + i] = tf32_rna(v - h);
    }
}

__global__ void split_kernel(const float *__restrict__ x, long long rows, int cols, long long ldx,
                             float *__restrict__ hi, float *__restrict__ lo, long long ldo) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= rows * cols) return;
    long long r = idx / cols;
    int c = int(idx % cols);
    float v = x[r * ldx + c];
    float h = tf32_rna(v);
    hi[r * ldo + c] = h;
    lo[r * ldo + c] = tf32_rna(v - h);
}

// Vectorized split for 16-byte aligned rows whose length is a multiple of 4.
__global__ void split4_kernel(const float4 *__restrict__ x, long long rows, int cols4,
                              long long ldx4, float4 *__restrict__ hi, float4 *__restrict__ lo,
                              long long ldo4) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= rows * cols4) return;
    long long r = idx / cols4;
    int c = int(idx % cols4);
    float4 v = x[r * ldx4 + c];
    float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
    float4 l = make_float4(tf32_rna(v.x - h.x), tf32_rna(v.y - h.y), tf32_rna(v.z - h.z),
                           tf32_rna(v.w - h.w));
    hi[r * ldo4 + c] = h;
    lo[r * ldo4 + c] = l;
}

// MSE upstream gradient: dY = (Y - T) * scale, split into TF32 planes; per-block
// sums of (Y - T)^2 in double (fixed reduction tree, deterministic).
__global__ void __launch_bounds__(256) mse_kernel(const float *__restrict__ y,
                                                  const float *__restrict__ t, long long rows,
                                                  int cols, long long ld, float scale,
                                                  float *__restrict__ hi, float *__restrict__ lo,
                                                  long long ldo, double *__restrict__ partial) {
    __shared__ double red[256];
    long long total = rows * cols;
    double acc = 0;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        long long r = idx / cols;
        int c = int(idx % cols);
        float d = y[r * ld + c] - t[r * ld + c];
        acc += double(d) * double(d);
        float g = d * scale;
        float h = tf32_rna(g);
        hi[r * ldo + c] = h;
        lo[r * ldo + c] = tf32_rna(g - h);
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

} // namespace tcst

using namespace tcst;

static int sm_count() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (count <= 0) count = 148;
    }
    return count;
}

extern "C" int tcst_assemble_weight(const void *atom_table_dev, int64_t atoms,
                                    const tcst_axis *out_axis, const tcst_axis *in_axis,
                                    int64_t *accumulator_dev, float *weight_dev,
                                    int64_t ld_weight, float *weight_hi_dev, float *weight_lo_dev,
                                    int64_t ld_split, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (atoms < 0 || !accumulator_dev || (atoms && !atom_table_dev) ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    int words = record_words(oa.modes, ia.modes);
    if (atoms > 0) {
        long long warps_needed = atoms;
        long long blocks = (warps_needed + 7) / 8;
        long long cap = (long long)sm_count() * 16;
        if (blocks > cap) blocks = cap;
        weight_scatter_kernel<<<unsigned(blocks), 256, 0, st>>>(
            (const float *)atom_table_dev, words, atoms, oa, ia,
            (unsigned long long *)accumulator_dev);
        TCST_CUDA(cudaGetLastError());
    }
    long long total = (long long)oa.sites * ia.sites;
    weight_finalize_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(
        (unsigned long long *)accumulator_dev, oa.sites, ia.sites, weight_dev, ld_weight,
        weight_hi_dev, weight_lo_dev, ld_split);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_split_tf32(const float *x_dev, int64_t rows, int64_t cols, int64_t ld_x,
                               float *hi_dev, float *lo_dev, int64_t ld_out, void *stream) {
    if (rows < 0 || cols < 0) {
        tcst_set_error("tcst_split_tf32: negative size");
        return TCST_ERR_ARGUMENT;
    }
    if (rows * cols == 0) return TCST_OK;
    if (ld_x < cols || ld_out < cols || !x_dev || !hi_dev || !lo_dev) {
        tcst_set_error("tcst_split_tf32: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    bool vec = cols % 4 == 0 && ld_x % 4 == 0 && ld_out % 4 == 0 &&
               (reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(hi_dev) |
                reinterpret_cast<uintptr_t>(lo_dev)) % 16 == 0;
    if (vec) {
        long long total = rows * (cols / 4);
        split4_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(
            (const float4 *)x_dev, rows, int(cols / 4), ld_x / 4, (float4 *)hi_dev,
            (float4 *)lo_dev, ld_out / 4);
    } else {
        long long total = rows * cols;
        split_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(x_dev, rows, int(cols), ld_x,
                                                                   hi_dev, lo_dev, ld_out);
    }
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_mse_grad(const float *y_dev, const float *target_dev, int64_t rows,
                             int64_t cols, int64_t ld, float scale, float *dy_hi_dev,
                             float *dy_lo_dev, int64_t ld_out, double *loss_partial_dev,
                             int32_t *blocks, void *stream) {
    int nblocks = sm_count() * 2;
    if (blocks) *blocks = nblocks;
    if (rows < 0 || cols < 1 || ld < cols || ld_out < cols || !loss_partial_dev ||
        (rows && (!y_dev || !target_dev || !dy_hi_dev || !dy_lo_dev))) {
        tcst_set_error("tcst_mse_grad: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    mse_kernel<<<nblocks, 256, 0, (cudaStream_t)stream>>>(y_dev, target_dev, rows, int(cols), ld,
                                                          scale, dy_hi_dev, dy_lo_dev, ld_out,
                                                          loss_partial_dev);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

// ---------------------------------------------------------------------------
// Weight assembly without caller-provided scratch.
//
// Some callers cannot hand this library device memory for the accumulator:
// a plugin running inside a host framework whose allocator owns every device
// byte, or a fixed-footprint deployment that forbids allocation after start-up.
// For them the accumulator lives in a fixed array compiled into this library.
// Every GPU that loads the library holds the array until the process exits.
// ---------------------------------------------------------------------------

#include <mutex>

namespace {

constexpr long long STATIC_WEIGHT_SITES = 1LL << 20; // N_out * N_in limit (8 MiB of int64)
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned long long g_static_accumulator[STATIC_WEIGHT_SITES];

std::mutex g_static_mutex;
unsigned long long *g_static_ptr[MAX_DEVICES] = {};

// Host code must not pass g_static_accumulator itself to a kernel: in host code
// that name is only a stand-in. The device address comes from
// cudaGetSymbolAddress, taken once per device with that device current; the
// array is cleared once there, and every later call leaves it all-zero again.
int static_accumulator(cudaStream_t stream, unsigned long long **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return tcst_cuda_check(e, "cudaGetDevice");
    if (dev < 0 || dev >= MAX_DEVICES) {
        tcst_set_error("tcst_assemble_weight_static: device ordinal %d out of range", dev);
        return TCST_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_ptr[dev]) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_static_accumulator);
        if (e != cudaSuccess) return tcst_cuda_check(e, "cudaGetSymbolAddress");
        e = cudaMemsetAsync(ptr, 0, sizeof(g_static_accumulator), stream);
        if (e != cudaSuccess) return tcst_cuda_check(e, "cudaMemsetAsync");
        g_static_ptr[dev] = static_cast<unsigned long long *>(ptr);
    }
    *out = g_static_ptr[dev];
    return TCST_OK;
}

} // namespace

extern "C" int64_t tcst_static_weight_sites(void) { return STATIC_WEIGHT_SITES; }

extern "C" int tcst_assemble_weight_static(const void *atom_table_dev, int64_t atoms,
                                           const tcst_axis *out_axis, const tcst_axis *in_axis,
                                           float *weight_dev, int64_t ld_weight,
                                           float *weight_hi_dev, float *weight_lo_dev,
                                           int64_t ld_split, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if ((long long)oa.sites * ia.sites > STATIC_WEIGHT_SITES) {
        tcst_set_error("tcst_assemble_weight_static: N_out * N_in = %lld exceeds the built-in "
                       "accumulator of %lld sites; use tcst_assemble_weight with caller memory",
                       (long long)oa.sites * ia.sites, STATIC_WEIGHT_SITES);
        return TCST_ERR_UNSUPPORTED;
    }
    if (atoms < 0 || (atoms && !atom_table_dev) ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight_static: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    unsigned long long *acc = nullptr;
    if ((rc = static_accumulator(st, &acc))) return rc;
    int words = record_words(oa.modes, ia.modes);
    if (atoms > 0) {
        long long blocks = (atoms + 7) / 8;
        long long cap = (long long)sm_count() * 16;
        if (blocks > cap) blocks = cap;
        weight_scatter_kernel<<<unsigned(blocks), 256, 0, st>>>(
            (const float *)atom_table_dev, words, atoms, oa, ia, acc);
        TCST_CUDA(cudaGetLastError());
    }
    long long total = (long long)oa.sites * ia.sites;
    weight_finalize_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(
        acc, oa.sites, ia.sites, weight_dev, ld_weight, weight_hi_dev, weight_lo_dev, ld_split);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
