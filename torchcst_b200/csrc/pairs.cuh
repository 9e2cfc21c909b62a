// Owner-pair (Fourier) path of coarse atoms: launches used by the weight
// assembly (forward) and the pullback (backward). See pairs.cu.
#pragma once

#include "common.cuh"

namespace tcst {

// A window W[r0 : r0 + wr, c0 : c0 + wc] of the weight (r0, c0 multiples of the
// weight tile), or of G's rows in the pullback.
struct Window {
    int r0, c0, wr, wc;
};

// TF32 bit pattern of x (round to nearest, ties away): the hi term of the
// three-product split x ~ hi + lo, lo = rn_tf32(x - hi).
__device__ __forceinline__ unsigned tf32_bits(float x) {
    unsigned r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// D += A B for one m16n8k8 TF32 tile. Fragments (g = lane / 4, q = lane % 4):
// a = A[g][q], A[g+8][q], A[g][q+4], A[g+8][q+4]; b = B[q][g], B[q+4][g];
// d = D[g][2q], D[g][2q+1], D[g+8][2q], D[g+8][2q+1].
__device__ __forceinline__ void mma_tf32(float (&d)[4], const unsigned (&a)[4], const unsigned (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Nodes (first tiles of T sites, nn of them on an axis of n sites) whose F-site
// footprint covers some site of [t0, t0 + tl): `count` consecutive nodes from
// `first` (mod nn). Node a covers the tile iff t0 - F < a T <= t0 + tl - 1
// modulo n.
__host__ __device__ __forceinline__ int cover_nodes(int t0, int tl, int T, int F, int nn, int n,
                                                    int &first) {
    first = 0;
    if (F + tl - 1 >= n) return nn;
    const int x = t0 - F + 1;
    const int lo = x >= 0 ? (x + T - 1) / T : -((-x) / T);
    const int hi = (t0 + tl - 1) / T;
    const int cnt = hi - lo + 1;
    if (cnt >= nn) return nn;
    first = lo % nn;
    first += first < 0 ? nn : 0;
    return cnt;
}


// Sum over the images of one chart site of the PF footprint functions
// {1, cos 2 pi k j / F, sin 2 pi k j / F}: d is the site minus the footprint
// start (any integer), images j = d mod n, d mod n + n, ... < F on an axis of
// n sites. False when no image lies on the footprint.
__device__ __forceinline__ bool pair_basis(int d, int F, int n, float *phi) {
    int j = d % n;
    j += j < 0 ? n : 0;
#pragma unroll
    for (int f = 0; f < PF; ++f) phi[f] = 0.f;
    bool hit = false;
    for (; j < F; j += n) {
        hit = true;
        float s1, c1;
        sincospif(2.0f * float(j) / float(F), &s1, &c1);
        phi[0] += 1.f;
        float cp = 1.f, cc = c1, sp = 0.f, sc = s1;
#pragma unroll
        for (int k = 1; k <= 8; ++k) {
            phi[2 * k - 1] += cc;
            phi[2 * k] += sc;
            const float cn = fmaf(2.f * c1, cc, -cp), sn = fmaf(2.f * c1, sc, -sp);
            cp = cc;
            cc = cn;
            sp = sc;
            sc = sn;
        }
    }
    return hit;
}


// CTAs of a launch over (expansion level-bank, output node, chunk of
// cols_per_cta input sites): 0 without expansion level-banks.
long long expand_ctas(const BinGeom &g, int n_in, int cols_per_cta);

// C of every active pair, then R and the node flags of the expansion
// level-banks for the nodes and columns the window's gather reads (before that
// gather).
int pair_forward(const Table &tv, const AxisCfg &oa, const AxisCfg &ia, const Window &win,
                 cudaStream_t st);

// P = Phi^T G per output node with an active pair, over the band's rows (G
// holds chart rows [band.r0, band.r0 + band.wr), summed over split-K
// partials, leading dimension ldg), then the gradients of the atoms of active
// pairs.
int pair_backward(const Table &tv, const AxisCfg &oa, const AxisCfg &ia, const float *g_dev,
                  long long ldg, const Window &band, float4 *grad, cudaStream_t st);

} // namespace tcst
