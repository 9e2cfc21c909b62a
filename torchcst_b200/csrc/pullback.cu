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
// its bin can reach (first-site bin + the class reach - 1 sites on both axes),
// then
//   classes 0, 1 (footprints <= 16, <= 32): four / eight threads per atom,
//                                 site values from the table's site buffer;
//   classes 2, 3 (<= 64, <= 128): one CTA per bin, one warp per atom, lanes
//                                 over input sites, output-site values in
//                                 per-warp shared memory.
// Atoms of active owner pairs take the owner-pair projection (pairs.cu). The
// other coarse atoms (and every atom of an unbinned geometry): one CTA per atom
// walks the footprint in chunks, G from global memory. Every atom is reduced by
// one thread group, one warp (fixed xor tree) or one CTA (fixed tree), so the
// gradient is bitwise reproducible. A band of G's rows can stand in for G (the
// output-row sharding): rows outside it read as zero.

#include <algorithm>

#include "common.cuh"
#include "pairs.cuh"

namespace tcst {

// Site-class pullback CTAs: 128 threads (32 quads or 16 octets per pass), about
// the atoms a first-site bin holds in the first training steps; six CTAs fit
// per SM (75 registers), so the 1,024 bins of a 1024 x 1024 layer take little
// more than one wave (256 threads left most quads idle in three CTAs per SM).
constexpr int P0_THREADS = 128;
constexpr int PC_THREADS = 256;
constexpr int PC_WARPS = PC_THREADS / 32;

// Whether chart rows {(r + k) mod n : 0 <= k < w} (0 <= r < n) meet the band
// [b0, b0 + bn) (0 <= b0, b0 + bn <= n).
__device__ __forceinline__ bool rows_meet(int r, int w, int n, int b0, int bn) {
    if (bn >= n || w >= n) return true;
    const int e = r + w;
    if (e <= n) return r < b0 + bn && b0 < e;
    return r < b0 + bn || b0 < e - n;
}

// G_0 += G_1 + ... + G_{split-1}, in place (rows of ni valid columns).
__global__ void g_reduce_kernel(float *__restrict__ g, int no, int ni, long long ldg, int split,
                                long long split_stride) {
    pdl_wait();
    const long long total = (long long)no * ni;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / ni, c = i - r * ni;
        float *gp = g + r * ldg + c;
        float v = gp[0];
        for (int s = 1; s < split; ++s) v += gp[s * split_stride];
        gp[0] = v;
    }
}

__global__ void g_reduce4_kernel(float4 *__restrict__ g, int no, int ni4, long long ldg4,
                                 int split, long long split_stride4) {
    pdl_wait();
    const long long total = (long long)no * ni4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / ni4, c = i - r * ni4;
        float4 *gp = g + r * ldg4 + c;
        float4 v = gp[0];
        for (int s = 1; s < split; ++s) {
            const float4 w = gp[s * split_stride4];
            v.x += w.x, v.y += w.y, v.z += w.z, v.w += w.w;
        }
        gp[0] = v;
    }
}

// G window [W x W] at (R0, C0) with rows/columns wrapped modulo no / ni.
// Interior windows (no column wrap, 16-byte aligned rows) move float4s, four
// in flight per thread; windows that wrap past the last column use scalars.
template <int W, int PITCH>
__device__ __forceinline__ void stage_window(float *gw, int R0, int C0, int no, int ni,
                                             const float *__restrict__ g, long long ldg, int split,
                                             long long split_stride, int b0, int bn) {
    constexpr int W4 = (W + 3) / 4; // float4 columns per row (PITCH >= 4 * W4)
    static_assert(PITCH >= 4 * W4 && PITCH % 4 == 0, "window pitch");
    const bool vec = split == 1 && C0 + 4 * W4 <= ni && ldg % 4 == 0 && C0 % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(g) & 15) == 0;
    if (vec) {
        constexpr int N4 = W * W4;
        for (int i0 = threadIdx.x; i0 < N4; i0 += 4 * blockDim.x) {
            float4 v[4];
            int dst[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * blockDim.x;
                dst[u] = -1;
                if (i < N4) {
                    const int rl = i / W4, c4 = i - rl * W4;
                    int row = R0 + rl;
                    while (row >= no) row -= no;
                    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row >= b0 && row < b0 + bn)
                        v[u] = *reinterpret_cast<const float4 *>(g + (long long)(row - b0) * ldg +
                                                                 C0 + 4 * c4);
                    dst[u] = rl * PITCH + 4 * c4;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (dst[u] >= 0) *reinterpret_cast<float4 *>(gw + dst[u]) = v[u];
        }
        return;
    }
    constexpr int N = W * W;
    for (int i0 = threadIdx.x; i0 < N; i0 += 8 * blockDim.x) {
        float v[8];
        int dst[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u * blockDim.x;
            dst[u] = -1;
            v[u] = 0.f;
            if (i < N) {
                const int rl = i / W, cl = i - rl * W;
                int row = R0 + rl, col = C0 + cl;
                while (row >= no) row -= no;
                while (col >= ni) col -= ni;
                if (row >= b0 && row < b0 + bn) {
                    const float *gp = g + (long long)(row - b0) * ldg + col;
                    v[u] = gp[0];
                    for (int s = 1; s < split; ++s) v[u] += gp[s * split_stride];
                }
                dst[u] = rl * PITCH + cl;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (dst[u] >= 0) gw[dst[u]] = v[u];
    }
}

// Rows [r_lo, r_hi) x columns [c_lo, c_hi) of the G window at (R0, C0) (window
// coordinates, pitch PITCH); float4s when the rectangle's columns do not wrap.
template <int PITCH>
__device__ __forceinline__ void stage_rect(float *gw, int r_lo, int r_hi, int c_lo, int c_hi,
                                           int R0, int C0, int no, int ni,
                                           const float *__restrict__ g, long long ldg, int b0,
                                           int bn) {
    c_lo &= ~3;
    const int nr = r_hi - r_lo, n4 = (c_hi - c_lo + 3) >> 2;
    if (nr <= 0 || n4 <= 0) return;
    const bool vec = C0 + c_lo + 4 * n4 <= ni && c_lo + 4 * n4 <= PITCH && ldg % 4 == 0 &&
                     C0 % 4 == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0;
    if (vec) {
        const int n = nr * n4;
        for (int i0 = threadIdx.x; i0 < n; i0 += 4 * blockDim.x) {
            float4 v[4];
            int dst[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * blockDim.x;
                dst[u] = -1;
                if (i < n) {
                    const int rr = i / n4, c4 = i - rr * n4;
                    int row = R0 + r_lo + rr;
                    while (row >= no) row -= no;
                    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row >= b0 && row < b0 + bn)
                        v[u] = *reinterpret_cast<const float4 *>(g + (long long)(row - b0) * ldg +
                                                                 C0 + c_lo + 4 * c4);
                    dst[u] = (r_lo + rr) * PITCH + c_lo + 4 * c4;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (dst[u] >= 0) *reinterpret_cast<float4 *>(gw + dst[u]) = v[u];
        }
        return;
    }
    const int nc = c_hi - c_lo, n = nr * nc;
    for (int i0 = threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {
        float v[8];
        int dst[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u * blockDim.x;
            dst[u] = -1;
            if (i < n) {
                const int rr = i / nc, cc = i - rr * nc;
                int row = R0 + r_lo + rr, col = C0 + c_lo + cc;
                while (row >= no) row -= no;
                while (col >= ni) col -= ni;
                v[u] = row >= b0 && row < b0 + bn ? g[(long long)(row - b0) * ldg + col] : 0.f;
                dst[u] = (r_lo + rr) * PITCH + c_lo + cc;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (dst[u] >= 0) gw[dst[u]] = v[u];
    }
}

// Site classes (footprints of at most 4 LANES sites: class 0 with LANES = 4,
// class 1 with LANES = 8): one CTA per first-site tile; LANES threads per atom,
// each owning four of the input sites; the output-site values of the atom are
// spread over the group and shuffled per row; the group sums its partials in a
// fixed xor order.
template <int E, int LANES>
__global__ void __launch_bounds__(P0_THREADS) pullback_site_kernel(
    Table tv, int cls, int no, int ni, const float *__restrict__ g, long long ldg, int split,
    long long split_stride, int b0, int bn, float4 *__restrict__ grad) {
    pdl_wait();
    constexpr int RS = 4 * LANES; // the class reach
    static_assert(RS <= REACH, "site values stored for the whole reach");
    constexpr int W = E + RS - 1;
    // Row pitch: W + 1 for the quads; for octets a multiple of 4 that is 4 mod 32
    // banks apart, so the eight rows one instruction reads spread over banks.
    constexpr int PITCH = LANES == 4 ? W + 1 : (W + 3) / 4 * 4 + ((W + 3) / 4 % 8 == 0 ? 4 : 0);
    __shared__ __align__(16) float gw[W * PITCH];
    const int ct = tv.geom.tc[cls];
    const int tr = blockIdx.x / ct, tc = blockIdx.x - tr * ct;
    const int bin = tv.geom.base[cls] + blockIdx.x; // the class's bins, row-major by tile
    const int begin = tv.offsets[bin], end = tv.offsets[bin + 1];
    const int R0 = tr * E, C0 = tc * E;
    if (begin == end || !rows_meet(R0, W, no, b0, bn)) return;
    stage_window<W, PITCH>(gw, R0, C0, no, ni, g, ldg, split, split_stride, b0, bn);
    __syncthreads();
    const int lane = threadIdx.x & 31, q = lane & (LANES - 1);
    const int groups = blockDim.x / LANES;
    for (int k0 = begin; k0 < end; k0 += groups) {
        const int k = k0 + threadIdx.x / LANES;
        const bool live = k < end;
        long long a = 0;
        int4 span = make_int4(0, 0, 0, 0);
        float4 om = make_float4(0, 0, 0, 0), od = om, orr = om, im = om, id = om, ir = om;
        if (live) {
            a = tv.ids[k];
            span = tv.sspan[k];
            const float4 *sv = reinterpret_cast<const float4 *>(tv.sites + a * SITE_FLOATS);
            constexpr int V = REACH / 4; // float4s per stored value row
            om = sv[q], od = sv[V + q], orr = sv[2 * V + q];           // output rows 4q .. 4q+3
            im = sv[3 * V + q], id = sv[4 * V + q], ir = sv[5 * V + q]; // input columns 4q .. 4q+3
        }
        const int fo = span.y, fi = span.w;
        float cm[4] = {im.x, im.y, im.z, im.w}, cd[4] = {id.x, id.y, id.z, id.w},
              cr[4] = {ir.x, ir.y, ir.z, ir.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (4 * q + j >= fi) cm[j] = cd[j] = cr[j] = 0.f;
        const float *g0 = gw + (live ? (span.x - R0) * PITCH + (span.z - C0) + 4 * q : 0);
        // Row contractions of the thread's four columns with (m, dm/dmu,
        // dm/dR) of the output sites, then one dot with the column values.
        float h0[4] = {}, h1[4] = {}, h2[4] = {};
        const int base = lane & ~(LANES - 1);
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            const float vm = (r & 3) == 0 ? om.x : (r & 3) == 1 ? om.y : (r & 3) == 2 ? om.z : om.w;
            const float vd = (r & 3) == 0 ? od.x : (r & 3) == 1 ? od.y : (r & 3) == 2 ? od.z : od.w;
            const float vr = (r & 3) == 0 ? orr.x : (r & 3) == 1 ? orr.y : (r & 3) == 2 ? orr.z : orr.w;
            const float rm = __shfl_sync(0xffffffffu, vm, base | (r >> 2));
            const float rdmu = __shfl_sync(0xffffffffu, vd, base | (r >> 2));
            const float rdr = __shfl_sync(0xffffffffu, vr, base | (r >> 2));
            if (r < fo) {
                const float *grow = g0 + r * PITCH;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float gv = grow[j];
                    h0[j] = fmaf(gv, rm, h0[j]);
                    h1[j] = fmaf(gv, rdmu, h1[j]);
                    h2[j] = fmaf(gv, rdr, h2[j]);
                }
            }
        }
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            s_amp = fmaf(h0[j], cm[j], s_amp);
            s_mo = fmaf(h1[j], cm[j], s_mo);
            s_mi = fmaf(h0[j], cd[j], s_mi);
            s_r = fmaf(h2[j], cm[j], fmaf(h0[j], cr[j], s_r));
        }
#pragma unroll
        for (int off = 1; off < LANES; off <<= 1) {
            s_amp += __shfl_xor_sync(0xffffffffu, s_amp, off);
            s_mo += __shfl_xor_sync(0xffffffffu, s_mo, off);
            s_mi += __shfl_xor_sync(0xffffffffu, s_mi, off);
            s_r += __shfl_xor_sync(0xffffffffu, s_r, off);
        }
        if (live && q == 0) grad[a] = atom_chain(tv.rec + a * (long long)tv.words, s_amp, s_mo, s_mi, s_r);
    }
}

// Classes 1 and 2: one CTA per bin (first-site tile). The CTA stages the
// bounding box of its atoms' footprints inside the (E + RC - 1)-square G
// window, then each warp takes one atom at a time: output-site values
// (m, dm/dmu, dm/dR) go to the warp's shared rows, lanes own input sites, and
// each lane accumulates the three row contractions of its columns before the
// fixed xor tree. Site phases use a per-atom step 2/F (within an ulp of the
// forward's phase; the gradient tolerance is far wider).
template <int RC, int E>
__global__ void __launch_bounds__(PC_THREADS) pullback_class_kernel(
    Table tv, int cls, int no, int ni, const float *__restrict__ g, long long ldg, int split,
    long long split_stride, int b0, int bn, float4 *__restrict__ grad) {
    pdl_wait();
    constexpr int W = E + RC - 1;
    constexpr int PITCH = W + 1;
    constexpr int Q = RC / 32;
    extern __shared__ __align__(16) float sm[];
    float *gw = sm;
    const BinGeom &geo = tv.geom;
    const int nc = geo.tc[cls];
    const int tr = blockIdx.x / nc, tc = blockIdx.x - tr * nc;
    const int bin = geo.base[cls] + blockIdx.x;
    const int begin = tv.offsets[bin], end = tv.offsets[bin + 1];
    const int R0 = tr * E, C0 = tc * E;
    if (begin == end || !rows_meet(R0, W, no, b0, bn)) return;
    // Stage only the bounding box of the bin's footprints.
    __shared__ int box[4]; // row lo, row hi, col lo, col hi (window coordinates)
    if (threadIdx.x == 0) box[0] = box[2] = W, box[1] = box[3] = 0;
    __syncthreads();
    {
        int rlo = W, rhi = 0, clo = W, chi = 0;
        for (int k = begin + threadIdx.x; k < end; k += blockDim.x) {
            const int4 sp = tv.sspan[k];
            rlo = min(rlo, sp.x - R0);
            rhi = max(rhi, sp.x - R0 + sp.y);
            clo = min(clo, sp.z - C0);
            chi = max(chi, sp.z - C0 + sp.w);
        }
        if (rhi > rlo) {
            atomicMin(&box[0], rlo);
            atomicMax(&box[1], min(rhi, W));
            atomicMin(&box[2], clo);
            atomicMax(&box[3], min(chi, W));
        }
    }
    __syncthreads();
    if (split == 1) {
        stage_rect<PITCH>(gw, box[0], box[1], box[2], box[3], R0, C0, no, ni, g, ldg, b0, bn);
    } else {
        stage_window<W, PITCH>(gw, R0, C0, no, ni, g, ldg, split, split_stride, b0, bn);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float4 *rowv = reinterpret_cast<float4 *>(sm + W * PITCH) + warp * RC; // (m, dm/dmu, dm/dR, 0)
    const int aw = axis_words(8);
    long long a_next = begin + warp < end ? tv.ids[begin + warp] : 0;
    for (int k = begin + warp; k < end; k += PC_WARPS) {
        const long long a = a_next;
        if (k + PC_WARPS < end) a_next = tv.ids[k + PC_WARPS];
        const int4 span = tv.sspan[k];
        const float *rec = tv.rec + a * (long long)tv.words;
        const int fo = span.y, fi = span.w;
        {
            AxisCoef<8> ao;
            ao.load(rec + 4);
            const float step = 2.0f / float(fo);
            for (int r = lane; r < fo; r += 32) {
                const SiteVals v = ao.values_at(fmaf(float(r), step, ao.phase0));
                rowv[r] = make_float4(v.m, v.dmu, v.dR, 0.f);
            }
        }
        float mi[Q], dmi[Q], dri[Q];
        int cl[Q];
        {
            AxisCoef<8> ai;
            ai.load(rec + 4 + aw);
            const float step = 2.0f / float(max(fi, 1));
#pragma unroll
            for (int j = 0; j < Q; ++j) {
                // Lanes past the footprint re-read the footprint's last (staged)
                // column with zero weights.
                const int c = lane + 32 * j;
                mi[j] = dmi[j] = dri[j] = 0.f;
                cl[j] = span.z - C0 + min(c, max(fi, 1) - 1);
                if (c < fi) {
                    const SiteVals v = ai.values_at(fmaf(float(c), step, ai.phase0));
                    mi[j] = v.m;
                    dmi[j] = v.dmu;
                    dri[j] = v.dR;
                }
            }
        }
        __syncwarp();
        float h0[Q], h1[Q], h2[Q];
#pragma unroll
        for (int j = 0; j < Q; ++j) h0[j] = h1[j] = h2[j] = 0.f;
        const float *g0 = gw + (span.x - R0) * PITCH;
        const int nq = (fi + 31) >> 5; // column slots in use (warp-uniform)
#pragma unroll 4
        for (int r = 0; r < fo; ++r) {
            const float4 rv = rowv[r];
            const float *grow = g0 + r * PITCH;
#pragma unroll
            for (int j = 0; j < Q; ++j) {
                if (j < nq) {
                    const float gv = grow[cl[j]];
                    h0[j] = fmaf(gv, rv.x, h0[j]);
                    h1[j] = fmaf(gv, rv.y, h1[j]);
                    h2[j] = fmaf(gv, rv.z, h2[j]);
                }
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
        if (lane == 0) grad[a] = atom_chain(rec, s_amp, s_mo, s_mi, s_r);
        __syncwarp();
    }
}
template <int RC, int E> constexpr size_t class_smem() {
    return size_t(E + RC - 1) * (E + RC) * 4 + size_t(PC_WARPS) * RC * 16;
}

// Coarse classes: one CTA per atom. The footprint is walked in chunks of
// PW_CHUNK x PW_CHUNK sites whose site values are staged in shared memory;
// warps take rows, lanes take columns, G comes from global memory. The atoms
// are ids[*begin .. atoms) (bound read on the device).
constexpr int PW_THREADS = 256;
constexpr int PW_CHUNK = 256;

__global__ void __launch_bounds__(PW_THREADS) pullback_wide_kernel(
    Table tv, const int *__restrict__ begin_ptr, AxisCfg out_ax, AxisCfg in_ax,
    const float *__restrict__ g, long long ldg, int split, long long split_stride, int b0,
    int bn, float4 *__restrict__ grad) {
    pdl_wait();
    __shared__ float so[3][PW_CHUNK], si[3][PW_CHUNK];
    __shared__ float red[PW_THREADS / 32][4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int aw = axis_words(out_ax.modes);
    const int ni = in_ax.sites, no = out_ax.sites;
    const long long begin = *begin_ptr;
    for (long long k = begin + blockIdx.x; k < tv.atoms; k += gridDim.x) {
        const long long a = tv.ids[k];
        if (pair_active(tv.geom, tv.offsets, tv.bin_of[a])) continue; // owner-pair path
        const float *rec = tv.rec + a * (long long)tv.words;
        const float *ob = rec + 4;
        const float *ib = rec + 4 + aw;
        const int4 sp = tv.spans[a];
        const int fo = sp.y, fi = sp.w;
        if (fo > 0 && !rows_meet(sp.x, fo, no, b0, bn)) continue; // CTA-uniform
        float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
        for (int r0 = 0; r0 < fo; r0 += PW_CHUNK) {
            const int nr = min(PW_CHUNK, fo - r0);
            for (int c0 = 0; c0 < fi; c0 += PW_CHUNK) {
                const int nc = min(PW_CHUNK, fi - c0);
                __syncthreads();
                for (int j = threadIdx.x; j < nr; j += PW_THREADS) {
                    const SiteVals v = site_values(ob, out_ax.modes, r0 + j, fo);
                    so[0][j] = v.m;
                    so[1][j] = v.dmu;
                    so[2][j] = v.dR;
                }
                for (int j = threadIdx.x; j < nc; j += PW_THREADS) {
                    const SiteVals v = site_values(ib, in_ax.modes, c0 + j, fi);
                    si[0][j] = v.m;
                    si[1][j] = v.dmu;
                    si[2][j] = v.dR;
                }
                __syncthreads();
                for (int r = warp; r < nr; r += PW_THREADS / 32) {
                    int row = sp.x + r0 + r;
                    while (row >= no) row -= no;
                    if (row < b0 || row >= b0 + bn) continue; // warp-uniform
                    const float mo = so[0][r], dmo = so[1][r], dro = so[2][r];
                    const float *grow = g + (long long)(row - b0) * ldg;
                    float h0 = 0.f, h1 = 0.f, h2 = 0.f;
                    for (int cb = 0; cb < nc; cb += 128) {
                        float gv[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int c = cb + lane + 32 * u;
                            gv[u] = 0.f;
                            if (c < nc) {
                                int col = sp.z + c0 + c;
                                while (col >= ni) col -= ni;
                                const float *gp = grow + col;
                                gv[u] = gp[0];
                                for (int s = 1; s < split; ++s) gv[u] += gp[s * split_stride];
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int c = cb + lane + 32 * u;
                            if (c < nc) {
                                h0 = fmaf(gv[u], si[0][c], h0); // sum G m_in
                                h1 = fmaf(gv[u], si[1][c], h1); // sum G dm_in/dmu
                                h2 = fmaf(gv[u], si[2][c], h2); // sum G dm_in/dR
                            }
                        }
                    }
                    s_amp = fmaf(mo, h0, s_amp);
                    s_mo = fmaf(dmo, h0, s_mo);
                    s_mi = fmaf(mo, h1, s_mi);
                    s_r = fmaf(dro, h0, fmaf(mo, h2, s_r));
                }
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
            red[warp][0] = s_amp;
            red[warp][1] = s_mo;
            red[warp][2] = s_mi;
            red[warp][3] = s_r;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
            for (int w = 0; w < PW_THREADS / 32; ++w) {
                t0 += red[w][0];
                t1 += red[w][1];
                t2 += red[w][2];
                t3 += red[w][3];
            }
            grad[a] = atom_chain(rec, t0, t1, t2, t3);
        }
        __syncthreads(); // red and the staged values are reused by the next atom
    }
}

} // namespace tcst

using namespace tcst;

// The fine-class kernels for bins of E sites per side.
template <int E>
static int launch_classes(const Table &tv, const AxisCfg &oa, const AxisCfg &ia, float *g_dev,
                          int64_t ldg, int split, int64_t split_stride, int b0, int bn,
                          float4 *grad, cudaStream_t st, cudaStream_t st1, cudaStream_t st2,
                          cudaStream_t st3) {
    const BinGeom &geo = tv.geom;
    static bool configured = false;
    if (!configured) {
        TCST_CUDA(cudaFuncSetAttribute(pullback_class_kernel<64, E>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(class_smem<64, E>())));
        TCST_CUDA(cudaFuncSetAttribute(pullback_class_kernel<128, E>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(class_smem<128, E>())));
        configured = true;
    }
    TCST_CUDA(launch_pdl(pullback_site_kernel<E, 4>, dim3(unsigned(geo.tr[0] * geo.tc[0])),
                         dim3(P0_THREADS), 0, st, tv, 0, oa.sites, ia.sites, g_dev, ldg, split,
                         split_stride, b0, bn, grad));
    TCST_CUDA(cudaGetLastError());
    if (geo.nclass > 1) {
        TCST_CUDA(launch_pdl(pullback_site_kernel<E, 8>, dim3(unsigned(geo.tr[1] * geo.tc[1])),
                             dim3(P0_THREADS), 0, st1, tv, 1, oa.sites, ia.sites, g_dev, ldg,
                             split, split_stride, b0, bn, grad));
        TCST_CUDA(cudaGetLastError());
    }
    // The two cached classes on streams of their own: few atoms reach them early
    // in training, but later each takes as long as the site classes together.
    if (geo.nclass > 2) {
        TCST_CUDA(launch_pdl(pullback_class_kernel<64, E>, dim3(unsigned(geo.tr[2] * geo.tc[2])),
                             dim3(PC_THREADS), class_smem<64, E>(), st2, tv, 2, oa.sites, ia.sites,
                             g_dev, ldg, split, split_stride, b0, bn, grad));
        TCST_CUDA(cudaGetLastError());
    }
    if (geo.nclass > 3) {
        TCST_CUDA(launch_pdl(pullback_class_kernel<128, E>,
                             dim3(unsigned(geo.tr[3] * geo.tc[3])), dim3(PC_THREADS),
                             class_smem<128, E>(), st3, tv, 3, oa.sites, ia.sites, g_dev, ldg,
                             split, split_stride, b0, bn, grad));
        TCST_CUDA(cudaGetLastError());
    }
    return TCST_OK;
}

// Pullback of the chart rows [row0, row0 + rows) of G (stored from g_dev, row
// row0 first); with a partial band every atom's gradient is the part its
// footprint rows inside the band contribute, and atoms outside it get zero.
static int pullback(const char *name, const void *atom_table_dev, int64_t atoms,
                    const tcst_axis *out_axis, const tcst_axis *in_axis, float *g_dev,
                    int64_t ldg, int32_t split, int64_t split_stride, int64_t row0, int64_t rows,
                    float *grad_dev, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (rows < 0) rows = oa.sites;
    if (atoms < 0 || split < 1 || ldg < ia.sites || row0 < 0 || row0 + rows > oa.sites ||
        (split > 1 && split_stride < rows * ldg) ||
        (atoms && rows && (!atom_table_dev || !g_dev || !grad_dev)) ||
        reinterpret_cast<uintptr_t>(grad_dev) % 16 ||
        reinterpret_cast<uintptr_t>(atom_table_dev) % 16) {
        tcst_set_error("%s: invalid arguments", name);
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const bool full = row0 == 0 && rows == oa.sites;
    if (!full) TCST_CUDA(cudaMemsetAsync(grad_dev, 0, size_t(atoms) * 16, st));
    if (rows == 0) return TCST_OK;
    const int words = record_words(oa.modes, ia.modes);
    const Table tv = table_view(atom_table_dev, atoms, words, axis_geo(oa), axis_geo(ia));
    const BinGeom &geo = tv.geom;
    float4 *grad = reinterpret_cast<float4 *>(grad_dev);
    const int b0 = int(row0), bn = int(rows);
    if (split > 1) {
        // Every later read of G then costs one load instead of `split`.
        const bool vec = ia.sites % 4 == 0 && ldg % 4 == 0 && split_stride % 4 == 0 &&
                         reinterpret_cast<uintptr_t>(g_dev) % 16 == 0;
        if (vec) {
            TCST_CUDA(launch_pdl(g_reduce4_kernel, dim3(148 * 8), dim3(256), 0, st,
                                 reinterpret_cast<float4 *>(g_dev), bn, ia.sites / 4, ldg / 4,
                                 split, split_stride / 4));
        } else {
            TCST_CUDA(launch_pdl(g_reduce_kernel, dim3(148 * 8), dim3(256), 0, st, g_dev, bn,
                                 ia.sites, ldg, split, split_stride));
        }
        TCST_CUDA(cudaGetLastError());
        split = 1;
    }
    // The class kernels, the owner-pair kernels and the wide kernel write
    // disjoint atoms' gradients: they run side by side on four side streams
    // beside the class-0 kernel (class 3 ahead of the wide kernel on the fourth),
    // joined before returning.
    SideStreams side(st, 4);
    if ((rc = side.status())) return rc;
    if (geo.nclass > 0) {
        rc = geo.fe == TS ? launch_classes<TS>(tv, oa, ia, g_dev, ldg, split, split_stride, b0,
                                               bn, grad, st, side[0], side[1], side[3])
                          : launch_classes<2 * TS>(tv, oa, ia, g_dev, ldg, split, split_stride,
                                                   b0, bn, grad, st, side[0], side[1], side[3]);
    }
    // Atoms of active owner pairs (their grads), then coarse classes, inactive
    // pair bins and invalid atoms (all atoms when unbinned): their range starts
    // at the first coarse bin and runs to the end of the ids.
    if (!rc) rc = pair_backward(tv, oa, ia, g_dev, ldg, Window{b0, 0, bn, ia.sites}, grad, side[2]);
    if (!rc) {
        const int first_bin = geo.nclass > 0 ? geo.base[std::min(NFINE, geo.nclass)] : 0;
        const long long ctas = std::min<long long>(atoms, 148LL * 8);
        const cudaError_t e = launch_pdl(pullback_wide_kernel, dim3(unsigned(ctas)),
                                         dim3(PW_THREADS), 0, side[3], tv, tv.offsets + first_bin,
                                         oa, ia, g_dev, ldg, split, split_stride, b0, bn, grad);
        if (e != cudaSuccess) rc = tcst_cuda_check(e, "pullback_wide_kernel");
    }
    const int rj = side.join();
    return rc ? rc : rj;
}

extern "C" int tcst_pullback(const void *atom_table_dev, int64_t atoms, const tcst_axis *out_axis,
                             const tcst_axis *in_axis, float *g_dev, int64_t ldg,
                             int32_t split, int64_t split_stride, float *grad_dev, void *stream) {
    return pullback("tcst_pullback", atom_table_dev, atoms, out_axis, in_axis, g_dev, ldg,
                          split, split_stride, 0, -1, grad_dev, stream);
}

extern "C" int tcst_pullback_band(const void *atom_table_dev, int64_t atoms,
                                  const tcst_axis *out_axis, const tcst_axis *in_axis,
                                  float *g_dev, int64_t ldg, int32_t split, int64_t split_stride,
                                  int64_t row0, int64_t rows, float *grad_dev, void *stream) {
    if (rows < 0) {
        tcst_set_error("tcst_pullback_band: negative row count");
        return TCST_ERR_ARGUMENT;
    }
    return pullback("tcst_pullback_band", atom_table_dev, atoms, out_axis, in_axis, g_dev,
                          ldg, split, split_stride, row0, rows, grad_dev, stream);
}
