// Atom-parameter gradient from G = dY^T X (summed over GEMM split-K partials).
//
// One warp per atom. Lanes own footprint columns (input sites); for each column
// a lane folds the footprint rows into three running row-sums
//   h0 = sum_r G m_out(r),  h1 = sum_r G dm_out/dmu(r),  h2 = sum_r G dm_out/dR(r)
// and then into the four atom sums
//   d amp = sum h0 m_in,  d mu_out/amp = sum h1 m_in,
//   d mu_in/amp = sum h0 dm_in/dmu,  d R/amp = sum (h2 m_in + h0 dm_in/dR).
// The warp reduction is a fixed xor tree, so the result is bitwise
// reproducible. The chain to (a, q) or (s, t) follows rational_radius.py:19-23
// and common.cuh:238-249 of the reference (Polar radii are detached).

#include "common.cuh"

namespace tcst {

__global__ void __launch_bounds__(256) pullback_kernel(
    const float *__restrict__ table, int words, long long atoms, AxisCfg out_ax, AxisCfg in_ax,
    const float *__restrict__ g, long long ldg, int split, long long split_stride,
    float4 *__restrict__ grad) {
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
        const int flags = reinterpret_cast<const int *>(rec)[3];
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
        if (fo > 0 && fi > 0) {
            const int first_o = reinterpret_cast<const int *>(ob)[0];
            const int first_i = reinterpret_cast<const int *>(ib)[0];
            for (int c0 = 0; c0 < fi; c0 += 32) {
                const int c = c0 + lane;
                const bool cv = c < fi;
                SiteVals vi = {0.f, 0.f, 0.f};
                if (cv) vi = site_values(ib, in_ax.modes, c, fi);
                const int col = wrap_site((long long)first_i + c, ni);
                float h0 = 0.f, h1 = 0.f, h2 = 0.f;
                for (int r0 = 0; r0 < fo; r0 += 32) {
                    const int rows = min(32, fo - r0);
                    SiteVals vo = {0.f, 0.f, 0.f};
                    if (lane < rows) vo = site_values(ob, out_ax.modes, r0 + lane, fo);
                    const int orow = wrap_site((long long)first_o + r0 + lane, no);
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
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            s_amp += __shfl_xor_sync(0xffffffffu, s_amp, off);
            s_mo += __shfl_xor_sync(0xffffffffu, s_mo, off);
            s_mi += __shfl_xor_sync(0xffffffffu, s_mi, off);
            s_r += __shfl_xor_sync(0xffffffffu, s_r, off);
        }
        if (lane == 0) {
            const float amp = rec[0], ch0 = rec[1], ch1 = rec[2];
            float4 out;
            if (flags & 2) {
                out = make_float4(0.f, 0.f, 0.f, 0.f);
            } else if (flags & 1) {
                // Polar: radius detached, amplitude chain to (s, t).
                out = make_float4(s_amp * ch0, s_amp * ch1, amp * s_mo, amp * s_mi);
            } else {
                const float d_r = amp * s_r;
                out = make_float4(fmaf(d_r, ch0, s_amp), d_r * ch1, amp * s_mo, amp * s_mi);
            }
            grad[a] = out;
        }
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
    int words = record_words(oa.modes, ia.modes);
    long long blocks = (atoms + 7) / 8;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    pullback_kernel<<<unsigned(blocks), 256, 0, (cudaStream_t)stream>>>(
        (const float *)atom_table_dev, words, atoms, oa, ia, g_dev, ldg, split, split_stride,
        (float4 *)grad_dev);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
