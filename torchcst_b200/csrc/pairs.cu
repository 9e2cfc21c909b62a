// Owner-pair (Fourier) path for coarse atoms that share an owner pair.
//
// All atoms of an owner pair (level-bank (T, K), output first tile a, input
// first tile b) share their footprints: F = K T sites from a T and from b T on
// the two axes. On a footprint the profile of an atom is a cosine series in the
// half-turn phase t_j = phase0 + 2 j / F (common.cuh), so with the PF = 2M + 1
// functions of the site j
//     phi_0 = 1, phi_{2k-1} = cos(2 pi k j / F), phi_{2k} = sin(2 pi k j / F)
// its mass is m(j) = sum_f alpha_f phi_f(j) with
//     alpha_0 = coef_0, alpha_{2k-1} = coef_k cos(pi k phase0),
//     alpha_{2k} = -coef_k sin(pi k phase0),
// and dm/dmu, dm/dR have coefficient vectors of the same form (below). The
// pair's contribution to W is therefore Phi_out C Phi_in^T with
//     C = sum_a amp_a alpha_out,a alpha_in,a^T          (PF x PF),
// and the pullback needs only H = Phi_out^T G Phi_in (PF x PF) per pair: every
// atom's four gradient sums are bilinear forms of H (this is the wide-atom
// factorisation of the reference's dense_fourier_weight.cuh and
// dense_pair_cotangent.cuh, restated). Sites past N fold onto the chart, so
// Phi is summed over the images of a chart site.
//
// Kernels (one launch each, all deterministic):
//   pair_coef_kernel     C of every active pair bin, atoms in bin (id) order;
//   pair_expand_kernel   per flagged output node a of an expansion level-bank
//                        and chunk of input sites: R_a = sum_b C_ab Phi_b^T
//                        (PF x N_in) over the active partners b in order; the
//                        weight gather then adds Phi_a(rows) R_a(cols) as PF
//                        rank-one terms per node (node flags and the count of
//                        active pairs come from the sort, atoms.cu);
//   pair_project_kernel  the pullback's P_a = Phi_a^T G (PF x N_in) per node
//                        with an active pair, over its footprint rows in order
//                        (a GEMM: tensor cores, three-product TF32);
//   pair_grad_kernel     per active pair H_ab = P_a Phi_b, then the gradient
//                        of each of its atoms.

#include <algorithm>

#include "pairs.cuh"

namespace tcst {

namespace {

constexpr int PC_CHUNK = 32;  // atoms staged per pass of pair_coef_kernel
constexpr int PC_THREADS = 96; // >= PF * PF4 accumulating threads and PC_CHUNK stagers
constexpr int PF4 = (PF + 3) / 4; // basis-length vectors as float4s (padded with zeros)
constexpr int PX_CHUNK = 256; // input sites per CTA of expand / project
constexpr int PG_COLS = 64;   // columns staged per pass of pair_grad_kernel

// Coefficient vectors of one axis block: m (alpha), dm/dmu (bmu), dm/dR (br).
//   dm/dmu(j) = omega sum_k k coef_k sin(pi k t_j)
//     -> bmu_{2k-1} = omega k coef_k sin(pi k phase0), bmu_{2k} = omega k coef_k cos(pi k phase0)
//   dm/dR(j) = sum_k dcoef_k cos(pi k t_j) -> br as alpha with dcoef.
__device__ __forceinline__ void axis_alpha(const float *blk, float *alpha, float *bmu,
                                           float *br) {
    const float p0 = blk[2], omega = blk[3];
    const float *c = blk + 4, *dc = blk + 4 + 9;
    float s1, c1;
    sincospif(p0, &s1, &c1);
    alpha[0] = c[0];
    if (bmu) bmu[0] = 0.f;
    if (br) br[0] = dc[0];
    float cp = 1.f, cc = c1, sp = 0.f, sc = s1;
#pragma unroll
    for (int k = 1; k <= 8; ++k) {
        alpha[2 * k - 1] = c[k] * cc;
        alpha[2 * k] = -c[k] * sc;
        if (bmu) {
            const float w = omega * float(k) * c[k];
            bmu[2 * k - 1] = w * sc;
            bmu[2 * k] = w * cc;
        }
        if (br) {
            br[2 * k - 1] = dc[k] * cc;
            br[2 * k] = -dc[k] * sc;
        }
        const float cn = fmaf(2.f * c1, cc, -cp), sn = fmaf(2.f * c1, sc, -sp);
        cp = cc;
        cc = cn;
        sp = sc;
        sc = sn;
    }
}

} // namespace

// Whether output node a of level-bank l covers a row of [r0, r0 + wr).
__device__ __forceinline__ bool node_covers(const BinGeom &g, int l, int a, int r0, int wr,
                                            int n_out) {
    int first;
    const int T = g.pl_T[l];
    const int cnt = cover_nodes(r0, wr, T, g.pl_K[l] * T, g.pl_no[l], n_out, first);
    int d = a - first;
    d += d < 0 ? g.pl_no[l] : 0;
    return d < cnt;
}

// Whether input node b of level-bank l covers a column of [c0, c0 + wc).
__device__ __forceinline__ bool in_node_covers(const BinGeom &g, int l, int b, int c0, int wc,
                                               int n_in) {
    int first;
    const int T = g.pl_T[l];
    const int cnt = cover_nodes(c0, wc, T, g.pl_K[l] * T, g.pl_ni[l], n_in, first);
    int d = b - first;
    d += d < 0 ? g.pl_ni[l] : 0;
    return d < cnt;
}

// C of the active pairs whose output node covers the window's rows and whose
// input node covers its columns (the only ones the window's expansion uses).
__global__ void __launch_bounds__(PC_THREADS) pair_coef_kernel(Table tv, int aw, int n_out,
                                                               int n_in, Window win) {
    pdl_wait();
    if (active_pairs(tv) == 0) return;
    const BinGeom &g = tv.geom;
    // amp alpha_out and alpha_in of PC_CHUNK atoms, rows padded to PF4 float4s.
    __shared__ float4 so[PC_CHUNK][PF4], si[PC_CHUNK][PF4];
    const int t = threadIdx.x;
    const int f = t / PF4, q = t - f * PF4; // C[f][4q .. 4q + 3] for t < PF * PF4
    const int pair_bins = g.pl_base[g.npl] - g.pl_base[0];
    for (int pb = blockIdx.x; pb < pair_bins; pb += gridDim.x) {
        const int bin = g.pl_base[0] + pb;
        if (!pair_active(g, tv.offsets, bin)) continue; // CTA-uniform
        {
            const int l = pair_lb(g, bin), idx = bin - g.pl_base[l];
            const int a = idx / g.pl_ni[l], b = idx - a * g.pl_ni[l];
            if (!node_covers(g, l, a, win.r0, win.wr, n_out) ||
                !in_node_covers(g, l, b, win.c0, win.wc, n_in))
                continue;
        }
        const int begin = tv.offsets[bin], end = tv.offsets[bin + 1];
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k0 = begin; k0 < end; k0 += PC_CHUNK) {
            const int n = min(PC_CHUNK, end - k0);
            if (t < n) {
                const long long a = tv.ids[k0 + t];
                const float *rec = tv.rec + a * (long long)tv.words;
                float ao[PF], ai[PF];
                axis_alpha(rec + 4, ao, nullptr, nullptr);
                axis_alpha(rec + 4 + aw, ai, nullptr, nullptr);
                const float amp = rec[0];
                float *po = reinterpret_cast<float *>(so[t]), *pi = reinterpret_cast<float *>(si[t]);
#pragma unroll
                for (int e = 0; e < 4 * PF4; ++e) {
                    po[e] = e < PF ? amp * ao[e] : 0.f;
                    pi[e] = e < PF ? ai[e] : 0.f;
                }
            }
            __syncthreads();
            if (t < PF * PF4)
                for (int j = 0; j < n; ++j) {
                    const float a = reinterpret_cast<const float *>(so[j])[f];
                    const float4 v = si[j][q];
                    acc[0] = fmaf(a, v.x, acc[0]);
                    acc[1] = fmaf(a, v.y, acc[1]);
                    acc[2] = fmaf(a, v.z, acc[2]);
                    acc[3] = fmaf(a, v.w, acc[3]);
                }
            __syncthreads();
        }
        if (t < PF * PF4) {
            float *out = tv.pair_c + (long long)pb * PF * PF + f * PF;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (4 * q + e < PF) out[4 * q + e] = acc[e];
        }
    }
}


// CTA -> (expansion level-bank l, output node a, input chunk ch).
__device__ __forceinline__ bool expand_cta(const BinGeom &g, int chunks, int &l, int &a,
                                           int &ch) {
    int cta = blockIdx.x;
    for (l = 0; l < g.npl; ++l) {
        if (!g.pl_exp[l]) continue;
        const int n = g.pl_no[l] * chunks;
        if (cta < n) break;
        cta -= n;
    }
    if (l >= g.npl) return false;
    a = cta / chunks;
    ch = cta - a * chunks;
    return true;
}


__global__ void __launch_bounds__(PX_CHUNK) pair_expand_kernel(Table tv, int n_out, int n_in,
                                                               Window win) {
    pdl_wait();
    const BinGeom &g = tv.geom;
    const int chunks = (n_in + PX_CHUNK - 1) / PX_CHUNK;
    int l, a, ch;
    if (active_pairs(tv) == 0 || !expand_cta(g, chunks, l, a, ch)) return;
    if (!tv.node_on[g.pl_node[l] + a]) return;
    // Only nodes over the window's rows and chunks over its columns are read
    // by the gather that follows (CTA-uniform exits).
    if (!node_covers(g, l, a, win.r0, win.wr, n_out)) return;
    if ((ch + 1) * PX_CHUNK <= win.c0 || ch * PX_CHUNK >= win.c0 + win.wc) return;
    const int T = g.pl_T[l], F = g.pl_K[l] * T, nb = g.pl_ni[l];
    const int i = ch * PX_CHUNK + threadIdx.x;
    __shared__ float4 C4[PF][PF4]; // C rows padded to float4s
    float r[PF];
#pragma unroll
    for (int f = 0; f < PF; ++f) r[f] = 0.f;
    for (int b = 0; b < nb; ++b) {
        const int bin = g.pl_base[l] + a * nb + b;
        if (tv.offsets[bin + 1] - tv.offsets[bin] < PAIR_MIN) continue; // CTA-uniform
        __syncthreads();
        for (int e = threadIdx.x; e < PF * 4 * PF4; e += blockDim.x) {
            const int f = e / (4 * PF4), k = e - f * (4 * PF4);
            reinterpret_cast<float *>(C4[f])[k] =
                k < PF ? tv.pair_c[(long long)(bin - g.pl_base[0]) * PF * PF + f * PF + k] : 0.f;
        }
        __syncthreads();
        float phi[4 * PF4];
        if (i < n_in && pair_basis(i - b * T, F, n_in, phi)) {
#pragma unroll
            for (int k = PF; k < 4 * PF4; ++k) phi[k] = 0.f;
#pragma unroll
            for (int f = 0; f < PF; ++f) {
                float v = r[f];
#pragma unroll
                for (int q = 0; q < PF4; ++q) {
                    const float4 c = C4[f][q];
                    v = fmaf(c.x, phi[4 * q], v);
                    v = fmaf(c.y, phi[4 * q + 1], v);
                    v = fmaf(c.z, phi[4 * q + 2], v);
                    v = fmaf(c.w, phi[4 * q + 3], v);
                }
                r[f] = v;
            }
        }
    }
    if (i < n_in) {
        float *out = tv.pair_buf + g.pl_buf[l] + (long long)a * PF * n_in + i;
#pragma unroll
        for (int f = 0; f < PF; ++f) out[(long long)f * n_in] = r[f];
    }
}

// G holds chart rows [band.r0, band.r0 + band.wr) at gm + (row - band.r0) ldg.
// P_a = Phi_a^T G is a GEMM (PF x rows times rows x N_in) per node: it runs on
// the tensor cores as mma.sync m16n8k8 TF32 with the three-product split of
// both operands (hi*hi + hi*lo + lo*hi, float32 accumulation), which keeps the
// float32 accuracy of the scalar form. A CTA owns PP_COLS input columns of one
// node; per chunk of PP_ROWS footprint rows it stages the basis values
// (transposed, PF padded to 32 with zeros) and the G block in shared memory,
// then each of the 8 warps multiplies the 32 x PP_ROWS basis block by its 32
// columns (2 x 4 tiles of 16 x 8). The row order of the sum is fixed, so P is
// deterministic.
constexpr int PP_COLS = 256;
constexpr int PP_ROWS = 32;
constexpr int PP_THREADS = 256;
constexpr int PP_GPITCH = PP_COLS + 8; // shared G row pitch (conflict-free fragment loads)
constexpr int PP_APITCH = 32 + 8;      // shared basis row pitch (conflict-free fragment loads)

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    const int n = valid ? 16 : 0; // a zero source size fills the 16 bytes with zeros
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

struct ProjectSmem {
    float sa[2][PP_ROWS][PP_APITCH]; // basis: [row][f], f >= PF zero
    float sg[2][PP_ROWS][PP_GPITCH]; // G block: [row][column]
};

__global__ void __launch_bounds__(PP_THREADS) pair_project_kernel(Table tv, int n_out, int n_in,
                                                                const float *__restrict__ gm,
                                                                long long ldg, Window band) {
    pdl_wait();
    const BinGeom &g = tv.geom;
    const int chunks = (n_in + PP_COLS - 1) / PP_COLS;
    int l, a, ch;
    if (active_pairs(tv) == 0 || !expand_cta(g, chunks, l, a, ch)) return;
    if (!tv.node_on[g.pl_node[l] + a] || !node_covers(g, l, a, band.r0, band.wr, n_out)) return;
    const int T = g.pl_T[l], F = g.pl_K[l] * T;
    const int c0 = ch * PP_COLS;
    // Rows to walk: the distinct chart rows of the footprint (all rows when it
    // wraps onto itself) or the band's rows, whichever is fewer; rows outside
    // the other set contribute zero.
    const int foot_rows = F >= n_out ? n_out : F;
    const bool by_band = band.wr < foot_rows;
    const int rows = by_band ? band.wr : foot_rows;
    const int row0 = by_band ? band.r0 : (F >= n_out ? 0 : a * T);
    extern __shared__ __align__(16) unsigned char pp_smem[];
    ProjectSmem &sm = *reinterpret_cast<ProjectSmem *>(pp_smem);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int gq = lane >> 2, tq = lane & 3; // fragment coordinates
    const int wc = warp * 32;                // the warp's first column in the CTA
    const bool vec = (ldg & 3) == 0 && (reinterpret_cast<uintptr_t>(gm) & 15) == 0;
    float acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
    // Stage chunk r0 into buffer b: basis values by warp 0 (one row per lane),
    // the G block by every thread (asynchronous 16-byte copies; rows outside
    // the band or footprint and columns past N_in fill with zeros).
    auto stage = [&](int r0, int b) {
        const int nr = min(PP_ROWS, rows - r0);
        if (warp == 0) {
            float phi[PF];
            int row = row0 + r0 + lane;
            row -= row >= n_out ? n_out : 0;
            const bool in = lane < nr && row >= band.r0 && row < band.r0 + band.wr &&
                            pair_basis(row - a * T, F, n_out, phi);
#pragma unroll
            for (int f = 0; f < 32; ++f) sm.sa[b][lane][f] = in && f < PF ? phi[f] : 0.f;
        }
        // Whether each staged row is in the band and on the footprint, per
        // thread (the rule pair_basis applies for warp 0's basis values).
        for (int i = t; i < PP_ROWS * (PP_COLS / 4); i += PP_THREADS) {
            const int r = i / (PP_COLS / 4), c4 = i - r * (PP_COLS / 4);
            int row = row0 + r0 + r;
            row -= row >= n_out ? n_out : 0;
            bool in = r < nr && row >= band.r0 && row < band.r0 + band.wr;
            if (in && F < n_out) { // on the footprint: (row - a T) mod n_out < F
                int d = (row - a * T) % n_out;
                d += d < 0 ? n_out : 0;
                in = d < F;
            }
            const int col = c0 + 4 * c4;
            float *dst = &sm.sg[b][r][4 * c4];
            const float *src = gm + (long long)(in ? row - band.r0 : 0) * ldg + (col < n_in ? col : 0);
            if (vec && col + 4 <= n_in) {
                cp_async16(dst, src, in);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    dst[e] = in && col + e < n_in ? gm[(long long)(row - band.r0) * ldg + col + e] : 0.f;
            }
        }
        cp_async_commit();
    };
    const int nchunks = (rows + PP_ROWS - 1) / PP_ROWS;
    stage(0, 0);
    for (int k = 0; k < nchunks; ++k) {
        const int b = k & 1;
        if (k + 1 < nchunks) {
            stage((k + 1) * PP_ROWS, b ^ 1);
            cp_async_wait1();
        } else {
            cp_async_wait0();
        }
        __syncthreads(); // chunk k staged (basis writes and copies) for every warp
#pragma unroll
        for (int k0 = 0; k0 < PP_ROWS; k0 += 8) {
            // A fragments (rows f = m, columns = footprint rows k), both m tiles.
            unsigned ah[2][4], al[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const float av[4] = {sm.sa[b][k0 + tq][mt * 16 + gq], sm.sa[b][k0 + tq][mt * 16 + gq + 8],
                                     sm.sa[b][k0 + tq + 4][mt * 16 + gq],
                                     sm.sa[b][k0 + tq + 4][mt * 16 + gq + 8]};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    ah[mt][e] = tf32_bits(av[e]);
                    al[mt][e] = tf32_bits(av[e] - __uint_as_float(ah[mt][e]));
                }
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int col = wc + nt * 8 + gq;
                const float bv[2] = {sm.sg[b][k0 + tq][col], sm.sg[b][k0 + tq + 4][col]};
                unsigned bh[2], bl[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    bh[e] = tf32_bits(bv[e]);
                    bl[e] = tf32_bits(bv[e] - __uint_as_float(bh[e]));
                }
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    mma_tf32(acc[mt][nt], al[mt], bh);
                    mma_tf32(acc[mt][nt], ah[mt], bl);
                    mma_tf32(acc[mt][nt], ah[mt], bh);
                }
            }
        }
        __syncthreads(); // buffer b is free for chunk k + 2
    }
    // Accumulator (m = f, n = column): c0 (gq, 2tq), c1 (gq, 2tq+1), c2 (gq+8, 2tq), c3 (gq+8, 2tq+1).
    float *out = tv.pair_buf + g.pl_buf[l] + (long long)a * PF * n_in;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int f = mt * 16 + gq + (e >= 2 ? 8 : 0);
                const int i = c0 + wc + nt * 8 + 2 * tq + (e & 1);
                if (f < PF && i < n_in) out[(long long)f * n_in + i] = acc[mt][nt][e];
            }
}

__global__ void __launch_bounds__(320) pair_grad_kernel(Table tv, int aw, int n_out, int n_in,
                                                        Window band, float4 *__restrict__ grad) {
    pdl_wait();
    if (active_pairs(tv) == 0) return;
    const BinGeom &g = tv.geom;
    __shared__ float sp[PF][PG_COLS + 1];
    __shared__ float4 sphi[PG_COLS][PF4]; // basis rows padded to float4s
    __shared__ float H[PF * PF];
    const int t = threadIdx.x;
    const int f = t / PF4, q = t - f * PF4; // H[f][4q .. 4q + 3] for t < PF * PF4
    const int lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    const int pair_bins = g.pl_base[g.npl] - g.pl_base[0];
    for (int pb = blockIdx.x; pb < pair_bins; pb += gridDim.x) {
        const int bin = g.pl_base[0] + pb;
        if (!pair_active(g, tv.offsets, bin)) continue; // CTA-uniform
        const int l = pair_lb(g, bin);
        const int nb = g.pl_ni[l], idx = bin - g.pl_base[l];
        const int a = idx / nb, b = idx - a * nb;
        // Outside the band the pair's rows contribute nothing (zero gradient).
        if (!node_covers(g, l, a, band.r0, band.wr, n_out)) continue;
        const int T = g.pl_T[l], F = g.pl_K[l] * T;
        const int cols = F >= n_in ? n_in : F;
        const int col0 = F >= n_in ? 0 : b * T;
        const float *P = tv.pair_buf + g.pl_buf[l] + (long long)a * PF * n_in;
        // H = P_a Phi_b over the distinct chart columns of b's footprint.
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = 0; c0 < cols; c0 += PG_COLS) {
            const int nc = min(PG_COLS, cols - c0);
            __syncthreads();
            for (int e = t; e < PF * nc; e += blockDim.x) {
                const int ff = e / nc, j = e - ff * nc;
                int col = col0 + c0 + j;
                col -= col >= n_in ? n_in : 0;
                sp[ff][j] = P[(long long)ff * n_in + col];
            }
            if (t < nc) {
                float phi[PF];
                int col = col0 + c0 + t;
                col -= col >= n_in ? n_in : 0;
                pair_basis(col - b * T, F, n_in, phi);
                float *dst = reinterpret_cast<float *>(sphi[t]);
#pragma unroll
                for (int e = 0; e < 4 * PF4; ++e) dst[e] = e < PF ? phi[e] : 0.f;
            }
            __syncthreads();
            if (t < PF * PF4)
                for (int j = 0; j < nc; ++j) {
                    const float pv = sp[f][j];
                    const float4 v = sphi[j][q];
                    acc[0] = fmaf(pv, v.x, acc[0]);
                    acc[1] = fmaf(pv, v.y, acc[1]);
                    acc[2] = fmaf(pv, v.z, acc[2]);
                    acc[3] = fmaf(pv, v.w, acc[3]);
                }
        }
        if (t < PF * PF4) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (4 * q + e < PF) H[f * PF + 4 * q + e] = acc[e];
        }
        __syncthreads();
        // Every atom of the pair: one warp, lanes over rows f of H.
        const int begin = tv.offsets[bin], end = tv.offsets[bin + 1];
        for (int k = begin + warp; k < end; k += nw) {
            const long long atom = tv.ids[k];
            const float *rec = tv.rec + atom * (long long)tv.words;
            float ao[PF], mo[PF], ro[PF], ai[PF], mi[PF], ri[PF];
            axis_alpha(rec + 4, ao, mo, ro);
            axis_alpha(rec + 4 + aw, ai, mi, ri);
            float s_amp = 0.f, s_mo = 0.f, s_mi = 0.f, s_r = 0.f;
            if (lane < PF) {
                float h1 = 0.f, h2 = 0.f, h3 = 0.f;
#pragma unroll
                for (int e = 0; e < PF; ++e) {
                    const float hv = H[lane * PF + e];
                    h1 = fmaf(hv, ai[e], h1);
                    h2 = fmaf(hv, mi[e], h2);
                    h3 = fmaf(hv, ri[e], h3);
                }
                // Row `lane` of the output-side vectors (registers are indexed
                // statically, so select by a loop).
                float a_f = 0.f, m_f = 0.f, r_f = 0.f;
#pragma unroll
                for (int e = 0; e < PF; ++e)
                    if (e == lane) {
                        a_f = ao[e];
                        m_f = mo[e];
                        r_f = ro[e];
                    }
                s_amp = a_f * h1;
                s_mo = m_f * h1;
                s_mi = a_f * h2;
                s_r = fmaf(r_f, h1, a_f * h3);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                s_amp += __shfl_xor_sync(0xffffffffu, s_amp, off);
                s_mo += __shfl_xor_sync(0xffffffffu, s_mo, off);
                s_mi += __shfl_xor_sync(0xffffffffu, s_mi, off);
                s_r += __shfl_xor_sync(0xffffffffu, s_r, off);
            }
            if (lane == 0) grad[atom] = atom_chain(rec, s_amp, s_mo, s_mi, s_r);
        }
        __syncthreads(); // H and the staging buffers are reused by the next pair
    }
}

int pair_forward(const Table &tv, const AxisCfg &oa, const AxisCfg &ia, const Window &win,
                 cudaStream_t st) {
    const BinGeom &g = tv.geom;
    if (g.npl == 0 || tv.atoms == 0) return TCST_OK;
    const int pair_bins = g.pl_base[g.npl] - g.pl_base[0];
    const int aw = axis_words(oa.modes);
    const unsigned grid = unsigned(std::min<long long>(pair_bins, 148LL * 8));
    TCST_CUDA(launch_pdl(pair_coef_kernel, dim3(grid), dim3(PC_THREADS), 0, st, tv, aw,
                         oa.sites, ia.sites, win));
    TCST_CUDA(cudaGetLastError());
    const long long ctas = expand_ctas(g, ia.sites, PX_CHUNK);
    if (ctas > 0) {
        TCST_CUDA(launch_pdl(pair_expand_kernel, dim3(unsigned(ctas)), dim3(PX_CHUNK), 0, st, tv,
                             oa.sites, ia.sites, win));
        TCST_CUDA(cudaGetLastError());
    }
    return TCST_OK;
}

int pair_backward(const Table &tv, const AxisCfg &oa, const AxisCfg &ia, const float *g_dev,
                  long long ldg, const Window &band, float4 *grad, cudaStream_t st) {
    const BinGeom &g = tv.geom;
    if (g.npl == 0 || tv.atoms == 0) return TCST_OK;
    const long long ctas = expand_ctas(g, ia.sites, PP_COLS);
    if (ctas == 0) return TCST_OK;
    static bool configured = false;
    if (!configured) {
        TCST_CUDA(cudaFuncSetAttribute(pair_project_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(sizeof(ProjectSmem))));
        configured = true;
    }
    TCST_CUDA(launch_pdl(pair_project_kernel, dim3(unsigned(ctas)), dim3(PP_THREADS),
                         sizeof(ProjectSmem), st, tv,
                         oa.sites, ia.sites, g_dev, ldg, band));
    TCST_CUDA(cudaGetLastError());
    const int pair_bins = g.pl_base[g.npl] - g.pl_base[0];
    const unsigned grid = unsigned(std::min<long long>(pair_bins, 148LL * 4));
    TCST_CUDA(launch_pdl(pair_grad_kernel, dim3(grid), dim3(320), 0, st, tv,
                         axis_words(oa.modes), oa.sites, ia.sites, band, grad));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

long long expand_ctas(const BinGeom &g, int n_in, int cols_per_cta) {
    const long long chunks = (n_in + cols_per_cta - 1) / cols_per_cta;
    long long n = 0;
    for (int l = 0; l < g.npl; ++l)
        if (g.pl_exp[l]) n += g.pl_no[l] * chunks;
    return n;
}

} // namespace tcst
