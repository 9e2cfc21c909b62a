// Dense weight assembly W = sum_a amp_a m_out,a (x) m_in,a, the TF32 split and
// the fused MSE gradient.
//
// Weight assembly uses the bins that tcst_decode_route stored in the atom
// table (footprint class x first-site tile, atoms in id order inside a bin):
//   wide:   atoms of the wide bin (footprint above the largest class) add their
//           products into a 64-bit fixed-point plane (2^-40 units) with global
//           reductions; integer adds are exact, so the plane does not depend on
//           the order in which they land;
//   gather: one CTA per TS x TS weight tile walks, in a fixed order, every bin
//           whose atoms can reach the tile, keeps the atoms that do, stages
//           their masses on the tile's rows and columns in shared memory
//           (images folded modulo N) and accumulates the outer products in
//           registers (4 x 4 per thread). The tile adds the wide plane and
//           writes W and/or its TF32 split planes.
// Fixed scan order + id-ordered bins make W bitwise reproducible.

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace tcst {

constexpr float FIXED_SCALE = 1099511627776.0f; // 2^40
constexpr double FIXED_UNIT = 1.0 / 1099511627776.0;
constexpr int WT_THREADS = 64; // 8 x 8 threads, 4 x 4 outputs each
constexpr int WT_BATCH = 32;   // atoms staged per pass

__device__ __forceinline__ float tf32_rna(float x) {
    unsigned r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ void red_add_u64(unsigned long long *addr, long long v) {
    asm volatile("red.global.add.u64 [%0], %1;" ::"l"(addr), "l"((unsigned long long)v) : "memory");
}

__host__ __device__ inline long long plane_words64(int n_out, int n_in) {
    return (long long)n_out * n_in;
}

// Does the cyclic footprint [f, f + F) (mod n) meet sites [t0, t0 + tl)?
__device__ __forceinline__ bool window_hits(int f, int F, int t0, int tl, int n) {
    if (F >= n) return true;
    int d = t0 - f;
    if (d < 0) d += n;
    return d < F || d + tl > n;
}

// Folded mass of the atom at the tile site t0 + p: sum over footprint sites j
// with (f + j) mod n == t0 + p. `sv` (class 0) holds the first REACH masses.
template <bool SITES>
__device__ __forceinline__ float folded_mass(const float *blk, const float *sv, int f, int F,
                                             int site, int n) {
    int j = site - f;
    if (j < 0) j += n;
    float v = 0.f;
    if (SITES) {
        for (; j < F; j += n) v += sv[j];
    } else {
        if (j >= F) return 0.f;
        AxisCoef<8> ac;
        ac.load_mass(blk);
        for (; j < F; j += n) v += ac.mass(j);
    }
    return v;
}

struct GatherOut {
    const unsigned long long *plane; // wide-atom plane or NULL
    float *w, *hi, *lo;
    long long ldw, lds;
};

__device__ __forceinline__ void gather_range(const Table &tv, int begin, int end, bool class0,
                                             int R0, int TR, int no, int C0, int TC, int ni,
                                             float (&acc)[4][4], int *cand, float (*us)[TS],
                                             float (*vs)[TS], int *wcount) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int r0 = (t >> 3) * 4, c0 = (t & 7) * 4;
    const int aw = axis_words(8);
    for (int base = begin; base < end; base += WT_THREADS) {
        const int idx = base + t;
        bool hit = false;
        int a = -1;
        if (idx < end) {
            a = tv.ids[idx];
            const int4 sp = tv.spans[a];
            hit = window_hits(sp.x, sp.y, R0, TR, no) && window_hits(sp.z, sp.w, C0, TC, ni);
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) wcount[warp] = __popc(m);
        __syncthreads();
        const int n = wcount[0] + wcount[1];
        if (hit) cand[(warp ? wcount[0] : 0) + __popc(m & ((1u << lane) - 1u))] = a;
        __syncthreads();
        for (int h = 0; h < n; h += WT_BATCH) {
            const int nb = min(WT_BATCH, n - h);
            // Warp 0 stages amp * m_out on the tile rows, warp 1 m_in on the columns.
            for (int s2 = 0; s2 < nb; ++s2) {
                const int atom = cand[h + s2];
                const float *rec = tv.rec + (long long)atom * tv.words;
                const int4 sp = tv.spans[atom];
                float v = 0.f;
                if (warp == 0) {
                    if (lane < TR) {
                        const float *sv = tv.sites + (long long)atom * SITE_FLOATS;
                        v = class0 ? folded_mass<true>(rec + 4, sv, sp.x, sp.y, R0 + lane, no)
                                   : folded_mass<false>(rec + 4, sv, sp.x, sp.y, R0 + lane, no);
                        v *= rec[0];
                    }
                    us[s2][lane] = v;
                } else {
                    if (lane < TC) {
                        const float *sv = tv.sites + (long long)atom * SITE_FLOATS + 3 * REACH;
                        v = class0 ? folded_mass<true>(rec + 4 + aw, sv, sp.z, sp.w, C0 + lane, ni)
                                   : folded_mass<false>(rec + 4 + aw, sv, sp.z, sp.w, C0 + lane, ni);
                    }
                    vs[s2][lane] = v;
                }
            }
            __syncthreads();
            for (int s2 = 0; s2 < nb; ++s2) {
                const float4 u = *reinterpret_cast<const float4 *>(&us[s2][r0]);
                const float4 v = *reinterpret_cast<const float4 *>(&vs[s2][c0]);
                const float uu[4] = {u.x, u.y, u.z, u.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(uu[i], vv[j], acc[i][j]);
            }
            __syncthreads();
        }
    }
}

__global__ void __launch_bounds__(WT_THREADS) weight_gather_kernel(Table tv, int no, int ni,
                                                                   int tiles_c, GatherOut out) {
    __shared__ __align__(16) float us[WT_BATCH][TS];
    __shared__ __align__(16) float vs[WT_BATCH][TS];
    __shared__ int cand[WT_THREADS];
    __shared__ int wcount[2];
    const int tr = blockIdx.x / tiles_c, tc = blockIdx.x - tr * tiles_c;
    const int R0 = tr * TS, C0 = tc * TS;
    const int TR = min(TS, no - R0), TC = min(TS, ni - C0);
    float acc[4][4] = {};
    const BinGeom &g = tv.geom;
    if (g.rt > 0) {
        for (int c = 0; c < NCLASS; ++c) {
            const int span_tiles = (class_reach(c) - 1 + TS - 1) / TS;
            const int kr = min(g.rt, 1 + span_tiles + (no % TS != 0));
            const int kc = min(g.ct, 1 + span_tiles + (ni % TS != 0));
            for (int k = 0; k < kr; ++k) {
                int sr = tr - k;
                sr += sr < 0 ? g.rt : 0;
                for (int l = 0; l < kc; ++l) {
                    int sc = tc - l;
                    sc += sc < 0 ? g.ct : 0;
                    const int bin = (c * g.rt + sr) * g.ct + sc;
                    gather_range(tv, tv.offsets[bin], tv.offsets[bin + 1], c == 0, R0, TR, no, C0,
                                 TC, ni, acc, cand, us, vs, wcount);
                }
            }
        }
    }
    const bool wide = out.plane && tv.offsets[g.nbins] > tv.offsets[g.nbins - 1];
    const int r0 = (threadIdx.x >> 3) * 4, c0 = (threadIdx.x & 7) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = r0 + i;
        if (r >= TR) continue;
        const long long row = R0 + r;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = c0 + j;
            if (c >= TC) continue;
            const long long col = C0 + c;
            float v = acc[i][j];
            if (wide) v += float(double((long long)out.plane[row * ni + col]) * FIXED_UNIT);
            if (out.w) out.w[row * out.ldw + col] = v;
            if (out.hi) {
                const float h = tf32_rna(v);
                out.hi[row * out.lds + col] = h;
                out.lo[row * out.lds + col] = tf32_rna(v - h);
            }
        }
    }
}

// Wide-bin atoms: one warp per atom adds its elements into the fixed-point
// plane. The atoms are ids[range[0] .. range[1]) (bounds read on the device).
__global__ void __launch_bounds__(256) weight_wide_kernel(Table tv, const int *__restrict__ range,
                                                          AxisCfg out_ax, AxisCfg in_ax,
                                                          unsigned long long *__restrict__ plane) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (gridDim.x * (long long)blockDim.x) >> 5;
    const int aw = axis_words(out_ax.modes);
    const int ni = in_ax.sites, no = out_ax.sites;
    const long long begin = range[0], end = range[1];
    for (long long k = begin + warp; k < end; k += nwarps) {
        const long long a = tv.ids[k];
        const float *rec = tv.rec + a * (long long)tv.words;
        const float *ob = rec + 4;
        const float *ib = rec + 4 + aw;
        const int fo = reinterpret_cast<const int *>(ob)[1];
        const int fi = reinterpret_cast<const int *>(ib)[1];
        const int first_o = reinterpret_cast<const int *>(ob)[0];
        const int first_i = reinterpret_cast<const int *>(ib)[0];
        const float amp = rec[0];
        for (int r0 = 0; r0 < fo; r0 += 32) {
            const int rows = min(32, fo - r0);
            const float mo = lane < rows ? amp * site_mass(ob, out_ax.modes, r0 + lane, fo) : 0.f;
            int orow = (first_o + r0 + lane) % no;
            orow = orow < 0 ? orow + no : orow;
            for (int cb = 0; cb < fi; cb += 32) {
                const int c = cb + lane;
                const bool cv = c < fi;
                const float mi = cv ? site_mass(ib, in_ax.modes, c, fi) * FIXED_SCALE : 0.f;
                int col = (first_i + c) % ni;
                col = col < 0 ? col + ni : col;
                for (int rr = 0; rr < rows; ++rr) {
                    const float v = __shfl_sync(0xffffffffu, mo, rr) * mi;
                    const int row = __shfl_sync(0xffffffffu, orow, rr);
                    if (cv) red_add_u64(plane + (long long)row * ni + col, __float2ll_rn(v));
                }
            }
        }
    }
}

__global__ void split_kernel(const float *__restrict__ x, int cols, long long ldx,
                             float *__restrict__ hi, float *__restrict__ lo, long long ldo) {
    const long long r = blockIdx.y;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
        const float v = x[r * ldx + c];
        const float h = tf32_rna(v);
        hi[r * ldo + c] = h;
        lo[r * ldo + c] = tf32_rna(v - h);
    }
}

// Vectorized split for 16-byte aligned rows whose length is a multiple of 4.
__global__ void split4_kernel(const float4 *__restrict__ x, long long rows, int cols4,
                              long long ldx4, float4 *__restrict__ hi, float4 *__restrict__ lo,
                              long long ldo4) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= rows * cols4) return;
    long long r = idx / cols4;
    int c = int(idx - r * cols4);
    float4 v = x[r * ldx4 + c];
    float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
    float4 l = make_float4(tf32_rna(v.x - h.x), tf32_rna(v.y - h.y), tf32_rna(v.z - h.z),
                           tf32_rna(v.w - h.w));
    hi[r * ldo4 + c] = h;
    lo[r * ldo4 + c] = l;
}

// MSE upstream gradient: dY = (Y - T) * scale, split into TF32 planes; per-block
// sums of (Y - T)^2 in double (fixed reduction tree, deterministic). Each CTA
// owns whole rows; vector path when rows are 16-byte aligned multiples of 4.
__global__ void __launch_bounds__(256) mse_kernel(const float *__restrict__ y,
                                                  const float *__restrict__ t, long long rows,
                                                  int cols, long long ld, float scale,
                                                  float *__restrict__ hi, float *__restrict__ lo,
                                                  long long ldo, double *__restrict__ partial,
                                                  int vec) {
    __shared__ double red[256];
    double acc = 0;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        if (vec) {
            const float4 *yr = reinterpret_cast<const float4 *>(y + r * ld);
            const float4 *tr = reinterpret_cast<const float4 *>(t + r * ld);
            float4 *hr = reinterpret_cast<float4 *>(hi + r * ldo);
            float4 *lr = reinterpret_cast<float4 *>(lo + r * ldo);
            for (int c = threadIdx.x; c < cols / 4; c += blockDim.x) {
                const float4 a = yr[c], b = tr[c];
                const float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
                acc += double(d0) * d0 + double(d1) * d1 + double(d2) * d2 + double(d3) * d3;
                const float g0 = d0 * scale, g1 = d1 * scale, g2 = d2 * scale, g3 = d3 * scale;
                const float4 h = make_float4(tf32_rna(g0), tf32_rna(g1), tf32_rna(g2), tf32_rna(g3));
                hr[c] = h;
                lr[c] = make_float4(tf32_rna(g0 - h.x), tf32_rna(g1 - h.y), tf32_rna(g2 - h.z),
                                    tf32_rna(g3 - h.w));
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += blockDim.x) {
                const float d = y[r * ld + c] - t[r * ld + c];
                acc += double(d) * double(d);
                const float g = d * scale;
                const float h = tf32_rna(g);
                hi[r * ldo + c] = h;
                lo[r * ldo + c] = tf32_rna(g - h);
            }
        }
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

extern "C" int64_t tcst_weight_scratch_bytes(int64_t atoms, const tcst_axis *out_axis,
                                             const tcst_axis *in_axis) {
    if (atoms < 0 || !out_axis || !in_axis || out_axis->site_count < 1 || in_axis->site_count < 1)
        return -1;
    return plane_words64(out_axis->site_count, in_axis->site_count) * 8;
}

static int assemble(const void *atom_table_dev, int64_t atoms, const AxisCfg &oa,
                    const AxisCfg &ia, void *scratch, float *weight_dev, int64_t ld_weight,
                    float *weight_hi_dev, float *weight_lo_dev, int64_t ld_split,
                    cudaStream_t st) {
    const int words = record_words(oa.modes, ia.modes);
    const Table tv = table_view(atom_table_dev, atoms, words, oa.sites, ia.sites, oa.modes, ia.modes);
    unsigned long long *plane = static_cast<unsigned long long *>(scratch);
    // Wide atoms: the plane is cleared and filled first; the wide bin's bounds
    // are only known on the device, so the kernel reads them.
    TCST_CUDA(cudaMemsetAsync(plane, 0, plane_words64(oa.sites, ia.sites) * 8, st));
    if (atoms > 0) {
        const long long warps = std::min<long long>(atoms, sm_count() * 32LL);
        weight_wide_kernel<<<unsigned((warps + 7) / 8), 256, 0, st>>>(
            tv, tv.offsets + tv.geom.nbins - 1, oa, ia, plane);
        TCST_CUDA(cudaGetLastError());
    }
    const int tiles_r = (oa.sites + TS - 1) / TS, tiles_c = (ia.sites + TS - 1) / TS;
    GatherOut out = {plane, weight_dev, weight_hi_dev, weight_lo_dev, ld_weight, ld_split};
    weight_gather_kernel<<<unsigned(tiles_r * tiles_c), WT_THREADS, 0, st>>>(tv, oa.sites, ia.sites,
                                                                           tiles_c, out);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_assemble_weight(const void *atom_table_dev, int64_t atoms,
                                    const tcst_axis *out_axis, const tcst_axis *in_axis,
                                    void *scratch_dev, int64_t scratch_bytes, float *weight_dev,
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
    if (atoms < 0 || !scratch_dev || !atom_table_dev ||
        scratch_bytes < plane_words64(oa.sites, ia.sites) * 8 ||
        reinterpret_cast<uintptr_t>(scratch_dev) % 16 ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    return assemble(atom_table_dev, atoms, oa, ia, scratch_dev, weight_dev, ld_weight,
                    weight_hi_dev, weight_lo_dev, ld_split, (cudaStream_t)stream);
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
        if (rows > 65535) {
            tcst_set_error("tcst_split_tf32: unaligned rows limited to 65535");
            return TCST_ERR_UNSUPPORTED;
        }
        dim3 grid(unsigned((cols + 255) / 256), unsigned(rows));
        split_kernel<<<grid, 256, 0, st>>>(x_dev, int(cols), ld_x, hi_dev, lo_dev, ld_out);
    }
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_mse_grad(const float *y_dev, const float *target_dev, int64_t rows,
                             int64_t cols, int64_t ld, float scale, float *dy_hi_dev,
                             float *dy_lo_dev, int64_t ld_out, double *loss_partial_dev,
                             int32_t *blocks, void *stream) {
    const int nblocks = sm_count() * 4;
    if (blocks) *blocks = nblocks;
    if (rows < 0 || cols < 1 || ld < cols || ld_out < cols || !loss_partial_dev ||
        (rows && (!y_dev || !target_dev || !dy_hi_dev || !dy_lo_dev))) {
        tcst_set_error("tcst_mse_grad: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    const int vec =
        cols % 4 == 0 && ld % 4 == 0 && ld_out % 4 == 0 &&
        ((reinterpret_cast<uintptr_t>(y_dev) | reinterpret_cast<uintptr_t>(target_dev) |
          reinterpret_cast<uintptr_t>(dy_hi_dev) | reinterpret_cast<uintptr_t>(dy_lo_dev)) % 16) == 0;
    mse_kernel<<<nblocks, 256, 0, (cudaStream_t)stream>>>(y_dev, target_dev, rows, int(cols), ld,
                                                          scale, dy_hi_dev, dy_lo_dev, ld_out,
                                                          loss_partial_dev, vec);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

// ---------------------------------------------------------------------------
// Weight assembly without caller-provided scratch.
//
// Some callers cannot hand this library device memory for the assembly's
// scratch: a plugin running inside a host framework whose allocator owns every
// device byte, or a fixed-footprint deployment that forbids allocation after
// start-up. For them the scratch lives in a fixed array compiled into this
// library. Every GPU that loads the library holds the array until the process
// exits.
// ---------------------------------------------------------------------------

namespace {

constexpr long long STATIC_SCRATCH_BYTES = 32LL << 20; // 32 MiB
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned long long g_static_scratch[STATIC_SCRATCH_BYTES / 8];

std::mutex g_static_mutex;
void *g_static_ptr[MAX_DEVICES] = {};

// Host code must not pass g_static_scratch itself to a kernel: in host code that
// name is only a stand-in. The device address comes from cudaGetSymbolAddress,
// taken once per device with that device current; the array is cleared once
// there, and every later call leaves its bin counters at zero again.
int static_scratch(cudaStream_t stream, void **out) {
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
        e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess) return tcst_cuda_check(e, "cudaGetSymbolAddress");
        e = cudaMemsetAsync(ptr, 0, sizeof(g_static_scratch), stream);
        if (e != cudaSuccess) return tcst_cuda_check(e, "cudaMemsetAsync");
        g_static_ptr[dev] = ptr;
    }
    *out = g_static_ptr[dev];
    return TCST_OK;
}

} // namespace

extern "C" int64_t tcst_static_weight_scratch_bytes(void) { return STATIC_SCRATCH_BYTES; }

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
    if (plane_words64(oa.sites, ia.sites) * 8 > STATIC_SCRATCH_BYTES) {
        tcst_set_error("tcst_assemble_weight_static: a %d x %d weight needs %lld scratch bytes, "
                       "more than the built-in %lld; use tcst_assemble_weight",
                       oa.sites, ia.sites, plane_words64(oa.sites, ia.sites) * 8,
                       STATIC_SCRATCH_BYTES);
        return TCST_ERR_UNSUPPORTED;
    }
    if (atoms < 0 || !atom_table_dev ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight_static: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    void *scratch = nullptr;
    if ((rc = static_scratch(st, &scratch))) return rc;
    return assemble(atom_table_dev, atoms, oa, ia, scratch, weight_dev, ld_weight, weight_hi_dev,
                    weight_lo_dev, ld_split, st);
}
