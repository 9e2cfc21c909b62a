// Atom-parameter gradient from G = dY^T X (summed over GEMM split-K partials).
//
// For every atom a the pullback reduces G over the atom's footprint:
//   d amp    = sum G m_out m_in
//   d mu_out = amp sum G dm_out/dmu m_in
//   d mu_in  = amp sum G m_out dm_in/dmu
//   d R      = amp sum G (dm_out/dR m_in + m_out dm_in/dR)
// then applies the rational (a, q) chain (rational_radius.py:19-23) or, for Polar
// rows whose radius is detached, the amplitude chain only.
//
// The atoms come from the bins of the atom table. Each binned class has its
// own kernel: a CTA stages in shared memory the window of G that every atom of
// its tile(s) can reach (first-site tile + the class reach - 1 sites on both
// axes, split-K partials summed while loading), then
//   class 0 (footprints <= 16):  one thread per atom, site values from the
//                                 table's site buffer;
//   classes 1, 2 (<= 64, <= 128): one warp per atom, lanes over input sites,
//                                 output-site values in per-warp shared memory.
// Wide-bin atoms: one warp per atom reads G from global memory. Every atom is
// reduced by one thread or one warp with a fixed xor tree, so the gradient is
// bitwise reproducible.

#include <algorithm>

#include "common.cuh"

namespace tcst {

constexpr int P0_THREADS = 128;
constexpr int PC_THREADS = 256;
constexpr int PC_WARPS = PC_THREADS / 32;

__device__ __forceinline__ float4 chain(const float *rec, float s_amp, float s_mo, float s_mi,
                                        float s_r) {
    const int flags = reinterpret_cast<const int *>(rec)[3];
    const float amp = rec[0], ch0 = rec[1], ch1 = rec[2];
    if (flags & 2) return make_float4(0.f, 0.f, 0.f, 0.f);
    if (flags & 1) return make_float4(s_amp * ch0, s_amp * ch1, amp * s_mo, amp * s_mi);
    const float d_r = amp * s_r;
    return make_float4(fmaf(d_r, ch0, s_amp), d_r * ch1, amp * s_mo, amp * s_mi);
}

// G window [wr x wc] at (R0, C0) with rows/columns wrapped modulo no / ni.
__device__ __forceinline__ void stage_window(float *gw, int wr, int wc, int pitch, int R0, int C0,
                                             int no, int ni, const float *__restrict__ g,
                                             long long ldg, int split, long long split_stride) {
    for (int i = threadIdx.x; i < wr * wc; i += blockDim.x) {
        const int rl = i / wc, cl = i - rl * wc;
        int row = R0 + rl, col = C0 + cl;
        while (row >= no) row -= no;
        while (col >= ni) col -= ni;
        const float *gp = g + (long long)row * ldg + col;
        float v = gp[0];
        for (int s = 1; s < split; ++s) v += gp[s * split_stride];
        gw[rl * pitch + cl] = v;
    }
}

// Class 0: one CTA per first-site tile, one thread per atom.
__global__ void __launch_bounds__(P0_THREADS) pullback_class0_kernel(
    Table tv, int no, int ni, const float *__restrict__ g, long long ldg, int split,
    long long split_stride, float4 *__restrict__ grad) {
    constexpr int W = TS + REACH - 1;
    __shared__ float gw[W * W];
    const int ct = tv.geom.ct;
    const int tr = blockIdx.x / ct, tc = blockIdx.x - tr * ct;
    const int bin = blockIdx.x; // class 0 bins come first, row-major by tile
    const int begin = tv.offsets[bin], end = tv.offsets[bin + 1];
    if (begin == end) return;
    const int R0 = tr * TS, C0 = tc * TS;
    stage_window(gw, W, W, W, R0, C0, no, ni, g, ldg, split, split_stride);
    __syncthreads();
    for (int k = begin + threadIdx.x; k < end; k += blockDim.x) {
        const long long a = tv.ids[k];
        const int4 span = tv.spans[a];
        const float *sv = tv.sites + a * SITE_FLOATS;
        const float4 *iv = reinterpret_cast<const float4 *>(sv + 3 * REACH);
        float im[REACH], idmu[REACH], idr[REACH];
#pragma unroll
        for (int q = 0; q < REACH / 4; ++q) {
            const float4 m4 = iv[q], u4 = iv[REACH / 4 + q], r4 = iv[REACH / 2 + q];
            im[4 * q] = m4.x, im[4 * q + 1] = m4.y, im[4 * q + 2] = m4.z, im[4 * q + 3] = m4.w;
            idmu[4 * q] = u4.x, idmu[4 * q + 1] = u4.y, idmu[4 * q + 2] = u4.z,
            idmu[4 * q + 3] = u4.w;
            idr[4 * q] = r4.x, idr[4 * q + 1] = r4.y, idr[4 * q + 2] = r4.z, idr[4 * q + 3] = r4.w;
        }
        const int fo = span.y, fi = span.w;
#pragma unroll
        for (int c = 0; c < REACH; ++c)
            if (c >= fi) im[c] = idmu[c] = idr[c] = 0.f;
        const float *g0 = gw + (span.x - R0) * W + (span.z - C0);
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
        for (int r = 0; r < fo; ++r) {
            const float rm = sv[r], rdmu = sv[REACH + r], rdr = sv[2 * REACH + r];
            const float *grow = g0 + r * W;
#pragma unroll
            for (int c = 0; c < REACH; ++c) {
                const float gv = c < fi ? grow[c] : 0.f;
                const float t = gv * im[c];
                const float u = gv * rm;
                s_amp = fmaf(t, rm, s_amp);
                s_mo = fmaf(t, rdmu, s_mo);
                s_mi = fmaf(u, idmu[c], s_mi);
                s_r = fmaf(t, rdr, fmaf(u, idr[c], s_r));
            }
        }
        grad[a] = chain(tv.rec + a * (long long)tv.words, s_amp, s_mo, s_mi, s_r);
    }
}

// Classes 1 and 2: one CTA per 2 x 2 block of first-site tiles, one warp per atom.
template <int RC>
__global__ void __launch_bounds__(PC_THREADS) pullback_class_kernel(
    Table tv, int cls, int no, int ni, const float *__restrict__ g, long long ldg, int split,
    long long split_stride, float4 *__restrict__ grad) {
    constexpr int W = 2 * TS + RC - 1;
    constexpr int PITCH = W + 1;
    constexpr int Q = RC / 32;
    extern __shared__ float sm[];
    float *gw = sm;
    const BinGeom &geo = tv.geom;
    const int rc2 = (geo.ct + 1) / 2;
    const int ir = blockIdx.x / rc2, ic = blockIdx.x - ir * rc2;
    int rb[4], re[4], total = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int tr = 2 * ir + (q >> 1), tc = 2 * ic + (q & 1);
        rb[q] = re[q] = 0;
        if (tr < geo.rt && tc < geo.ct) {
            const int bin = (cls * geo.rt + tr) * geo.ct + tc;
            rb[q] = tv.offsets[bin];
            re[q] = tv.offsets[bin + 1];
        }
        total += re[q] - rb[q];
    }
    if (total == 0) return;
    const int R0 = 2 * ir * TS, C0 = 2 * ic * TS;
    stage_window(gw, W, W, PITCH, R0, C0, no, ni, g, ldg, split, split_stride);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *rowv = sm + W * PITCH + warp * 3 * RC; // m, dm/dmu, dm/dR of the output sites
    const int aw = axis_words(8);
    for (int item = warp; item < total; item += PC_WARPS) {
        int k = item, q = 0;
        while (k >= re[q] - rb[q]) {
            k -= re[q] - rb[q];
            ++q;
        }
        const long long a = tv.ids[rb[q] + k];
        const int4 span = tv.spans[a];
        const float *rec = tv.rec + a * (long long)tv.words;
        const int fo = span.y, fi = span.w;
        {
            AxisCoef<8> ao;
            ao.load(rec + 4);
            for (int r = lane; r < fo; r += 32) {
                const SiteVals v = ao.values(r);
                rowv[r] = v.m;
                rowv[RC + r] = v.dmu;
                rowv[2 * RC + r] = v.dR;
            }
        }
        float mi[Q], dmi[Q], dri[Q];
        int cl[Q];
        {
            AxisCoef<8> ai;
            ai.load(rec + 4 + aw);
#pragma unroll
            for (int j = 0; j < Q; ++j) {
                const int c = lane + 32 * j;
                mi[j] = dmi[j] = dri[j] = 0.f;
                cl[j] = -1;
                if (c < fi) {
                    const SiteVals v = ai.values(c);
                    mi[j] = v.m;
                    dmi[j] = v.dmu;
                    dri[j] = v.dR;
                    cl[j] = span.z - C0 + c;
                }
            }
        }
        __syncwarp();
        float h0[Q], h1[Q], h2[Q];
#pragma unroll
        for (int j = 0; j < Q; ++j) h0[j] = h1[j] = h2[j] = 0.f;
        const float *g0 = gw + (span.x - R0) * PITCH;
        for (int r = 0; r < fo; ++r) {
            const float m = rowv[r], dm = rowv[RC + r], dr = rowv[2 * RC + r];
            const float *grow = g0 + r * PITCH;
#pragma unroll
            for (int j = 0; j < Q; ++j) {
                const float gv = cl[j] >= 0 ? grow[cl[j]] : 0.f;
                h0[j] = fmaf(gv, m, h0[j]);
                h1[j] = fmaf(gv, dm, h1[j]);
                h2[j] = fmaf(gv, dr, h2[j]);
            }
        }
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
#pragma unroll
        for (int j = 0; j < Q; ++j) {
            s_amp = fmaf(h0[j], mi[j], s_amp);
            s_mo = fmaf(h1[j], mi[j], s_mo);
            s_mi = fmaf(h0[j], dmi[j], s_mi);
            s_r = fmaf(h2[j], mi[j], fmaf(h0[j], dri[j], s_r));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            s_amp += __shfl_xor_sync(0xffffffffu, s_amp, off);
            s_mo += __shfl_xor_sync(0xffffffffu, s_mo, off);
            s_mi += __shfl_xor_sync(0xffffffffu, s_mi, off);
            s_r += __shfl_xor_sync(0xffffffffu, s_r, off);
        }
        if (lane == 0) grad[a] = chain(rec, s_amp, s_mo, s_mi, s_r);
        __syncwarp();
    }
}

template <int RC> constexpr size_t class_smem() {
    return size_t(2 * TS + RC - 1) * (2 * TS + RC) * 4 + size_t(PC_WARPS) * 3 * RC * 4;
}

// Wide-bin atoms: one warp per atom, G from global memory. The atoms are
// ids[range[0] .. range[1]) (bounds read on the device).
__global__ void __launch_bounds__(256) pullback_wide_kernel(
    Table tv, const int *__restrict__ range, AxisCfg out_ax, AxisCfg in_ax,
    const float *__restrict__ g, long long ldg, int split, long long split_stride,
    float4 *__restrict__ grad) {
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
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
        for (int cb = 0; cb < fi; cb += 32) {
            const int c = cb + lane;
            const bool cv = c < fi;
            SiteVals vi = {0.f, 0.f, 0.f};
            if (cv) vi = site_values(ib, in_ax.modes, c, fi);
            int col = (first_i + c) % ni;
            col = col < 0 ? col + ni : col;
            float h0 = 0.f, h1 = 0.f, h2 = 0.f;
            for (int r0 = 0; r0 < fo; r0 += 32) {
                const int rows = min(32, fo - r0);
                SiteVals vo = {0.f, 0.f, 0.f};
                if (lane < rows) vo = site_values(ob, out_ax.modes, r0 + lane, fo);
                int orow = (first_o + r0 + lane) % no;
                orow = orow < 0 ? orow + no : orow;
                for (int rr = 0; rr < rows; ++rr) {
                    const float mo = __shfl_sync(0xffffffffu, vo.m, rr);
                    const float dmo = __shfl_sync(0xffffffffu, vo.dmu, rr);
                    const float dro = __shfl_sync(0xffffffffu, vo.dR, rr);
                    const int row = __shfl_sync(0xffffffffu, orow, rr);
                    if (cv) {
                        const float *gp = g + (long long)row * ldg + col;
                        float gv = gp[0];
                        for (int s = 1; s < split; ++s) gv += gp[s * split_stride];
                        h0 = fmaf(gv, mo, h0);
                        h1 = fmaf(gv, dmo, h1);
                        h2 = fmaf(gv, dro, h2);
                    }
                }
            }
            s_amp = fmaf(h0, vi.m, s_amp);
            s_mo = fmaf(h1, vi.m, s_mo);
            s_mi = fmaf(h0, vi.dmu, s_mi);
            s_r = fmaf(h2, vi.m, fmaf(h0, vi.dR, s_r));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            s_amp += __shfl_xor_sync(0xffffffffu, s_amp, off);
            s_mo += __shfl_xor_sync(0xffffffffu, s_mo, off);
            s_mi += __shfl_xor_sync(0xffffffffu, s_mi, off);
            s_r += __shfl_xor_sync(0xffffffffu, s_r, off);
        }
        if (lane == 0) grad[a] = chain(rec, s_amp, s_mo, s_mi, s_r);
    }
}

} // namespace tcst

using namespace tcst;

extern "C" int tcst_pullback(const void *atom_table_dev, int64_t atoms, const tcst_axis *out_axis,
                             const tcst_axis *in_axis, const float *g_dev, int64_t ldg,
                             int32_t split, int64_t split_stride, float *grad_dev, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (atoms < 0 || split < 1 || ldg < ia.sites ||
        (split > 1 && split_stride < (long long)oa.sites * ldg) ||
        (atoms && (!atom_table_dev || !g_dev || !grad_dev)) ||
        reinterpret_cast<uintptr_t>(grad_dev) % 16) {
        tcst_set_error("tcst_pullback: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    const int words = record_words(oa.modes, ia.modes);
    const Table tv = table_view(atom_table_dev, atoms, words, oa.sites, ia.sites, oa.modes, ia.modes);
    const BinGeom &geo = tv.geom;
    cudaStream_t st = (cudaStream_t)stream;
    float4 *grad = reinterpret_cast<float4 *>(grad_dev);
    if (geo.rt > 0) {
        static bool configured = false;
        if (!configured) {
            TCST_CUDA(cudaFuncSetAttribute(pullback_class_kernel<64>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(class_smem<64>())));
            TCST_CUDA(cudaFuncSetAttribute(pullback_class_kernel<128>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(class_smem<128>())));
            configured = true;
        }
        pullback_class0_kernel<<<unsigned(geo.rt * geo.ct), P0_THREADS, 0, st>>>(
            tv, oa.sites, ia.sites, g_dev, ldg, split, split_stride, grad);
        TCST_CUDA(cudaGetLastError());
        const unsigned regions = unsigned(((geo.rt + 1) / 2) * ((geo.ct + 1) / 2));
        pullback_class_kernel<64><<<regions, PC_THREADS, class_smem<64>(), st>>>(
            tv, 1, oa.sites, ia.sites, g_dev, ldg, split, split_stride, grad);
        TCST_CUDA(cudaGetLastError());
        pullback_class_kernel<128><<<regions, PC_THREADS, class_smem<128>(), st>>>(
            tv, 2, oa.sites, ia.sites, g_dev, ldg, split, split_stride, grad);
        TCST_CUDA(cudaGetLastError());
    }
    const long long warps = std::min<long long>(atoms, 148LL * 32);
    pullback_wide_kernel<<<unsigned((warps + 7) / 8), 256, 0, st>>>(
        tv, tv.offsets + geo.nbins - 1, oa, ia, g_dev, ldg, split, split_stride, grad);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
