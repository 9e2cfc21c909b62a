// Dense weight assembly W = sum_a amp_a m_out,a (x) m_in,a (or a window of it),
// the f16 / TF32 splits and the MSE gradient.
//
// Weight assembly uses the bins that tcst_decode_route stored in the atom
// table (footprint class x first-site tile, or owner pair; atoms in id order
// inside a bin):
//   cache:  one warp per atom of classes SITE_CLASSES..NFINE-1 writes the atom's
//           masses on both footprints into the caller's scratch (the masses of
//           footprints of at most REACH sites are in the atom table's site
//           buffer; coarser classes are evaluated where used);
//   pairs:  the owner-pair coefficients and expansions (pairs.cu);
//   gather: one CTA per TS x TS weight tile lists, in a fixed order, every bin
//           whose atoms can reach the tile (active owner pairs excepted), keeps
//           the atoms that do, stages their masses on the tile's rows and
//           columns in shared memory as [site][hit] planes (images folded
//           modulo N; one thread per hit and axis) and accumulates the outer
//           products as a [32 x hits] x [hits x 32] product on the tensor cores
//           (mma.sync TF32, three-product split), adds the rank-one terms of the
//           active owner nodes that cover the tile the same way, then writes W
//           (or its TF32 split planes) and folds max |W| in.
// A fixed bin order and id-ordered bins make W bitwise reproducible; the only
// atomic is the max.

#include <algorithm>
#include <mutex>

#include <cuda_fp16.h>

#include "common.cuh"
#include "pairs.cuh"

namespace tcst {

constexpr int WT_THREADS = 128; // four warps, a 16 x 16 quarter of the tile each
constexpr int WT_STAGE = 56;    // hits staged per sub-pass (eight CTAs fit an SM)
constexpr int WT_KP = WT_STAGE + 4; // pitch of the staged [site][hit] planes: 60 = -4
                                    // (mod 32 banks), so the MMA fragment loads
                                    // (8 rows x 4 hits) hit 32 distinct banks
constexpr int MAX_SCAN = 512;  // bins a weight tile can scan

__device__ __forceinline__ float tf32_rna(float x) {
    unsigned r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__host__ __device__ inline long long cache_floats(long long atoms) {
    return atoms * 2 * CACHE_SITES;
}

// Does the cyclic footprint [f, f + F) (mod n) meet sites [t0, t0 + tl)?
__device__ __forceinline__ bool window_hits(int f, int F, int t0, int tl, int n) {
    if (F >= n) return true;
    int d = t0 - f;
    if (d < 0) d += n;
    return d < F || d + tl > n;
}

// Source tiles (k = 0 .. count-1 steps back from the tile holding `t0`) whose
// atoms of class c can reach sites [t0, t0 + TS).
__host__ __device__ __forceinline__ int reach_tiles(int c, int fe, int tiles, int n) {
    const int e = class_edge(c, fe);
    const int k = 1 + (class_reach(c) - 1 + e - 1) / e + (n % e != 0);
    return min(k, tiles);
}

// Upper bound of the bins one weight tile scans (class bins within reach and
// covering pair bins).
__host__ inline int max_scan_entries(const BinGeom &g, int no, int ni) {
    if (g.nclass == 0) return 1;
    int n = 0;
    for (int c = 0; c < g.nclass; ++c) n += reach_tiles(c, g.fe, g.tr[c], no) * reach_tiles(c, g.fe, g.tc[c], ni);
    for (int l = 0; l < g.npl; ++l) {
        const int k = g.pl_K[l] + 2;
        n += (g.pl_no[l] < k ? g.pl_no[l] : k) * (g.pl_ni[l] < k ? g.pl_ni[l] : k);
    }
    return n;
}

// Class SITE_CLASSES..NFINE-1 mass cache: cache[a][axis][j] = m_axis(j), j < F_axis.
__global__ void __launch_bounds__(256) mass_cache_kernel(Table tv, float *__restrict__ cache) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (gridDim.x * (long long)blockDim.x) >> 5;
    const BinGeom &g = tv.geom;
    const int begin = tv.offsets[g.base[min(SITE_CLASSES, g.nclass)]];
    const int end = tv.offsets[g.base[min(NFINE, g.nclass)]];
    const int aw = axis_words(8);
    const int side = lane >> 4, l = lane & 15; // half-warp per axis
    for (long long k = begin + warp; k < end; k += nwarps) {
        const long long a = tv.ids[k];
        const float *rec = tv.rec + a * (long long)tv.words;
        const int4 sp = tv.sspan[k];
        AxisCoef<8> ac;
        ac.load_mass(rec + 4 + side * aw);
        const int F = side ? sp.w : sp.y;
        float *dst = cache + (a * 2 + side) * CACHE_SITES;
        // cos / sin of pi t_j by rotation along the lane's sites j = l, l + 16, ...
        float sj, cj, sd, cd;
        sincospif(ac.phase0 + 2.0f * float(l) / float(F), &sj, &cj);
        sincospif(32.0f / float(F), &sd, &cd);
        for (int j = l; j < F; j += 16) {
            dst[j] = ac.mass_c(cj);
            const float cn = fmaf(cj, cd, -sj * sd);
            sj = fmaf(sj, cd, cj * sd);
            cj = cn;
        }
    }
}

// Per-tensor power-of-two scale of the F16 split: max |s X| lands in
// [2^14, 2^15), inside the f16 range with the hi rounding included.
__device__ __forceinline__ float f16_scale(float amax) {
    if (!(amax > 0.f) || !(amax < 3.0e38f)) return 1.f;
    int e;
    frexpf(amax, &e); // amax = m 2^e, m in [0.5, 1)
    const int k = max(-120, min(120, 15 - e));
    return ldexpf(1.f, k);
}

__device__ __forceinline__ void atomic_max_abs(float *amax, float v) {
    // Non-negative floats order like their bit patterns.
    atomicMax(reinterpret_cast<unsigned *>(amax), __float_as_uint(v));
}

// Block-wide max of m (blockDim.x <= 1024, a multiple of 32), then one atomic
// per block: same-address atomics serialize, so keep them few.
__device__ __forceinline__ void block_max_to(float *amax, float m) {
    __shared__ float wmax[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0 && m > 0.f) atomic_max_abs(amax, m);
    }
}

struct GatherOut {
    float *w, *hi, *lo;
    long long ldw, lds;
    float *amax; // nullable: max |W| folded in, one atomic per tile
    // Window W[r0 : r0 + wr, c0 : c0 + wc] (r0, c0 multiples of TS); W[r][c]
    // is stored at (r - r0, c - c0).
    int r0, c0, wr, wc;
};

// acc += U V^T over the staged hits [0, kpad) (kpad a multiple of 8; the
// planes are zero past the staged hits): U = us [tile row][hit], V = vs [tile
// column][hit]. Warp w owns rows 16 (w / 2) .. +15 and columns 16 (w % 2) ..
// +15 (two n-tiles). Three-product TF32 split (lo hi + hi lo + hi hi), so the
// products keep about 22 significant bits, accumulated in fp32.
__device__ __forceinline__ void tile_mma(float (&acc)[2][4], const float (*us)[WT_KP],
                                         const float (*vs)[WT_KP], int kpad, int warp, int lane) {
    const int g = lane >> 2, q = lane & 3;
    const int m0 = (warp >> 1) * 16, n0 = (warp & 1) * 16;
#pragma unroll 2
    for (int k0 = 0; k0 < kpad; k0 += 8) {
        const float av[4] = {us[m0 + g][k0 + q], us[m0 + g + 8][k0 + q], us[m0 + g][k0 + q + 4],
                             us[m0 + g + 8][k0 + q + 4]};
        unsigned ah[4], al[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            ah[e] = tf32_bits(av[e]);
            al[e] = tf32_bits(av[e] - __uint_as_float(ah[e]));
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const int c = n0 + nt * 8 + g;
            const float bv[2] = {vs[c][k0 + q], vs[c][k0 + q + 4]};
            unsigned bh[2], bl[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                bh[e] = tf32_bits(bv[e]);
                bl[e] = tf32_bits(bv[e] - __uint_as_float(bh[e]));
            }
            mma_tf32(acc[nt], al, bh);
            mma_tf32(acc[nt], ah, bl);
            mma_tf32(acc[nt], ah, bh);
        }
    }
}

// Zero columns [0, kpad) of both staged planes (kpad a multiple of 4).
__device__ __forceinline__ void zero_planes(float (*us)[WT_KP], float (*vs)[WT_KP], int kpad,
                                            int t) {
    const int per_row = kpad >> 2, per_plane = TS * per_row;
    for (int e = t; e < 2 * per_plane; e += WT_THREADS) {
        const int pl = e >= per_plane, rem = e - pl * per_plane;
        const int r = rem / per_row, c4 = rem - r * per_row;
        float(*dst)[WT_KP] = pl ? vs : us;
        *reinterpret_cast<float4 *>(&dst[r][4 * c4]) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

__global__ void __launch_bounds__(WT_THREADS, 8) weight_gather_kernel(Table tv, int no, int ni,
                                                                   int modes_o, int modes_i,
                                                                   int tiles_c,
                                                                   const float *__restrict__ cache,
                                                                   GatherOut out) {
    pdl_wait();
    __shared__ int sbeg[MAX_SCAN], scls[MAX_SCAN], spre[MAX_SCAN + 1];
    __shared__ int wtot[WT_THREADS / 32];
    // Staged hits: us[r][h] = amp_h m_out,h at tile row r, vs[c][h] = m_in,h at
    // tile column c (images folded modulo N), zero off the footprints.
    __shared__ __align__(16) float us[TS][WT_KP];
    __shared__ __align__(16) float vs[TS][WT_KP];
    __shared__ int cand[WT_THREADS], ccls[WT_THREADS];
    __shared__ int4 cspan[WT_THREADS];
    __shared__ float camp[WT_THREADS];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int trow = blockIdx.x / tiles_c, tcol = blockIdx.x - trow * tiles_c;
    const int R0 = out.r0 + trow * TS, C0 = out.c0 + tcol * TS;
    const int TR = min(TS, out.r0 + out.wr - R0), TC = min(TS, out.c0 + out.wc - C0);
    const BinGeom &g = tv.geom;

    // 1. The bins to scan, in a fixed order, with their atom counts.
    int nscan;
    if (g.nclass == 0) {
        nscan = 1;
        if (t == 0) {
            sbeg[0] = tv.offsets[0];
            scls[0] = -1;
            spre[0] = 0;
            spre[1] = tv.offsets[1] - tv.offsets[0];
        }
    } else {
        // Groups: the classes (their bins within reach), then the level-banks
        // (the pair bins of covering node pairs; active pairs count no atoms:
        // they come in as rank-one terms below). One thread per group finds
        // its covering rows and columns, warp 0 forms the prefix over groups,
        // and every entry then finds its group by bisection. Group
        // descriptors and prefix borrow cspan / ccls, free until step 2.
        static_assert(MAX_CLASSES + MAX_PAIR_LB <= 64, "groups: two per lane of warp 0");
        static_assert(MAX_CLASSES + MAX_PAIR_LB <= WT_THREADS && 65 <= WT_THREADS,
                      "group descriptors and prefix fit cspan / ccls");
        const int ngroups = g.nclass + g.npl;
        int4 *gdesc = cspan;                  // (first row, first column, columns, entries)
        int *gpre = ccls;
        if (t < ngroups) {
            int cr, cc, fr, fc, first_bin, end_bin;
            if (t < g.nclass) {
                // Class edges are powers of two: the tile holding R0 by a shift.
                const int sh = 31 - __clz(class_edge(t, g.fe));
                cr = reach_tiles(t, g.fe, g.tr[t], no);
                cc = reach_tiles(t, g.fe, g.tc[t], ni);
                fr = R0 >> sh;
                fc = C0 >> sh;
                first_bin = g.base[t], end_bin = g.base[t + 1];
            } else {
                const int l = t - g.nclass, T = g.pl_T[l], F = g.pl_K[l] * T;
                cr = cover_nodes(R0, TR, T, F, g.pl_no[l], no, fr);
                cc = cover_nodes(C0, TC, T, F, g.pl_ni[l], ni, fc);
                first_bin = g.pl_base[l], end_bin = g.pl_base[l + 1];
            }
            // A group without atoms (early in training most classes are empty)
            // contributes no scan entries.
            const bool empty = tv.offsets[first_bin] == tv.offsets[end_bin];
            gdesc[t] = make_int4(fr, fc, cc, empty ? 0 : cr * cc);
        }
        __syncthreads();
        if (warp == 0) {
            int lo = lane < ngroups ? gdesc[lane].w : 0;
            int hi = lane + 32 < ngroups ? gdesc[lane + 32].w : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y0 = __shfl_up_sync(0xffffffffu, lo, o);
                const int y1 = __shfl_up_sync(0xffffffffu, hi, o);
                if (lane >= o) {
                    lo += y0;
                    hi += y1;
                }
            }
            const int lo_total = __shfl_sync(0xffffffffu, lo, 31);
            gpre[lane + 1] = lo;
            gpre[lane + 33] = lo_total + hi;
            if (lane == 0) gpre[0] = 0;
        }
        __syncthreads();
        nscan = gpre[ngroups];
        for (int i = t; i < nscan; i += WT_THREADS) {
            int lo = 0, hi = ngroups - 1; // last group with gpre[k] <= i
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (gpre[mid] <= i) lo = mid;
                else hi = mid - 1;
            }
            const int4 d = gdesc[lo];
            const int rem = i - gpre[lo], u = rem / d.z, v = rem - u * d.z;
            if (lo < g.nclass) {
                const int c = lo;
                int sr = d.x - u, sc = d.y - v;
                sr += sr < 0 ? g.tr[c] : 0;
                sc += sc < 0 ? g.tc[c] : 0;
                const int bin = g.base[c] + sr * g.tc[c] + sc;
                sbeg[i] = tv.offsets[bin];
                spre[i + 1] = tv.offsets[bin + 1] - sbeg[i];
                scls[i] = c;
            } else {
                const int l = lo - g.nclass, F = g.pl_K[l] * g.pl_T[l];
                const int a = d.x + u >= g.pl_no[l] ? d.x + u - g.pl_no[l] : d.x + u;
                const int b = d.y + v >= g.pl_ni[l] ? d.y + v - g.pl_ni[l] : d.y + v;
                const int bin = g.pl_base[l] + a * g.pl_ni[l] + b;
                sbeg[i] = tv.offsets[bin];
                spre[i + 1] = pair_active(g, tv.offsets, bin) ? 0 : tv.offsets[bin + 1] - sbeg[i];
                scls[i] = atom_class(make_int4(0, F, 0, F));
            }
        }
        __syncthreads();
        // Inclusive prefix of the counts in spre[1..nscan], contiguous runs per thread.
        const int per = (nscan + WT_THREADS - 1) / WT_THREADS, i0 = t * per;
        int local = 0;
        for (int k = 0; k < per; ++k)
            if (i0 + k < nscan) local += spre[i0 + k + 1];
        int inc = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) wtot[warp] = inc;
        __syncthreads();
        int run = inc - local;
        for (int w = 0; w < warp; ++w) run += wtot[w];
        for (int k = 0; k < per; ++k)
            if (i0 + k < nscan) {
                run += spre[i0 + k + 1];
                spre[i0 + k + 1] = run;
            }
        if (t == 0) spre[0] = 0;
    }
    __syncthreads();
    const int total = spre[nscan];
    const int aw = axis_words(modes_o);
    float acc[2][4] = {};

    // 2. Candidates in passes of one per thread: keep those that reach the tile.
    for (int base = 0; base < total; base += WT_THREADS) {
        const int i = base + t;
        bool hit = false;
        int a = 0, cls = 0;
        float amp = 0.f;
        int4 sp = make_int4(0, 0, 0, 0);
        if (i < total) {
            int lo = 0, hi = nscan - 1; // last slot with spre[slot] <= i
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (spre[mid] <= i) lo = mid;
                else hi = mid - 1;
            }
            const int k = sbeg[lo] + (i - spre[lo]);
            a = tv.ids[k];
            cls = scls[lo];
            sp = tv.sspan[k];
            amp = tv.samp[k];
            hit = window_hits(sp.x, sp.y, R0, TR, no) && window_hits(sp.z, sp.w, C0, TC, ni);
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) wtot[warp] = __popc(m);
        __syncthreads();
        int n = 0, before = 0;
#pragma unroll
        for (int w = 0; w < WT_THREADS / 32; ++w) {
            before += w < warp ? wtot[w] : 0;
            n += wtot[w];
        }
        if (hit) {
            const int slot = before + __popc(m & ((1u << lane) - 1u));
            cand[slot] = a;
            ccls[slot] = cls;
            cspan[slot] = sp;
            camp[slot] = amp;
        }
        __syncthreads();
        for (int h0 = 0; h0 < n; h0 += WT_STAGE) {
            const int nb = min(WT_STAGE, n - h0), kpad = (nb + 7) & ~7;
            zero_planes(us, vs, kpad, t);
            __syncthreads();
            // 3. Stage, one thread per (hit, axis): warps 0-1 the rows (amp m_out),
            // warps 2-3 the columns (m_in). Classes with stored masses and a
            // footprint of at most N sites (one image per tile site) write the
            // covered sites, at most two runs of the cyclic footprint; the other
            // hits are evaluated in a second pass (one lane per tile site).
            bool rest = false;
            {
                const int side = t >> 6, s2 = t & 63;
                if (s2 < nb) {
                    const int4 qs = cspan[h0 + s2];
                    const int f = side ? qs.z : qs.x, F = side ? qs.w : qs.y;
                    const int c = ccls[h0 + s2];
                    const int nn = side ? ni : no, lim = side ? TC : TR;
                    if (c >= 0 && c < NFINE && F <= nn) {
                        const long long atom = cand[h0 + s2];
                        const float *src = c < SITE_CLASSES ? tv.sites + atom * SITE_FLOATS + side * 3 * REACH
                                                  : cache + (atom * 2 + side) * CACHE_SITES;
                        const float scale = side ? 1.f : camp[h0 + s2];
                        float(*dst)[WT_KP] = side ? vs : us;
                        // Footprint index of tile site 0 (f and the tile origin lie in
                        // [0, N)); tile sites [0, F - j0) and [N - j0, N - j0 + F).
                        int j0 = (side ? C0 : R0) - f;
                        j0 += j0 < 0 ? nn : 0;
                        const int a_end = j0 < F ? min(lim, F - j0) : 0;
                        const int b0 = nn - j0, b_end = min(lim, b0 + F);
                        // Eight independent loads in flight per chunk.
                        for (int r0 = 0; r0 < a_end; r0 += 8) {
                            float v[8];
#pragma unroll
                            for (int u = 0; u < 8; ++u) v[u] = r0 + u < a_end ? src[j0 + r0 + u] : 0.f;
#pragma unroll
                            for (int u = 0; u < 8; ++u)
                                if (r0 + u < a_end) dst[r0 + u][s2] = scale * v[u];
                        }
                        for (int r0 = b0; r0 < b_end; r0 += 8) {
                            float v[8];
#pragma unroll
                            for (int u = 0; u < 8; ++u) v[u] = r0 + u < b_end ? src[r0 + u - b0] : 0.f;
#pragma unroll
                            for (int u = 0; u < 8; ++u)
                                if (r0 + u < b_end) dst[r0 + u][s2] = scale * v[u];
                        }
                    } else {
                        rest = true;
                    }
                }
            }
            if (__syncthreads_or(rest)) {
                const int side = warp >> 1, sub = warp & 1;
                const int lim = side ? TC : TR, nn = side ? ni : no;
                const int p = lane, site = (side ? C0 : R0) + p;
                float(*dst)[WT_KP] = side ? vs : us;
                for (int s2 = sub; s2 < nb; s2 += 2) {
                    const int4 qs = cspan[h0 + s2];
                    const int f = side ? qs.z : qs.x, F = side ? qs.w : qs.y;
                    const int c = ccls[h0 + s2];
                    if (c >= 0 && c < NFINE && F <= nn) continue;
                    const long long atom = cand[h0 + s2];
                    int j = site - f;
                    j += j < 0 ? nn : 0;
                    float v = 0.f;
                    if (p < lim && j < F) {
                        const float *blk = tv.rec + atom * tv.words + 4 + side * aw;
                        if (c >= 0 && c < SITE_CLASSES) {
                            const float *sv = tv.sites + atom * SITE_FLOATS + side * 3 * REACH;
                            for (; j < F; j += nn) v += sv[j];
                        } else if (c >= SITE_CLASSES && c < NFINE) {
                            const float *cv = cache + (atom * 2 + side) * CACHE_SITES;
                            for (; j < F; j += nn) v += cv[j];
                        } else if (c >= NFINE) {
                            AxisCoef<8> ac;
                            ac.load_mass(blk);
                            for (; j < F; j += nn) v += ac.mass(j);
                        } else {
                            // Unbinned geometry: any mode count.
                            const int modes = side ? modes_i : modes_o;
                            for (; j < F; j += nn) v += site_mass(blk, modes, j, F);
                        }
                    }
                    if (p < TS) dst[p][s2] = side ? v : v * camp[h0 + s2];
                }
                __syncthreads();
            }
            tile_mma(acc, us, vs, kpad, warp, lane);
            __syncthreads();
        }
    }

    // 4. Active owner pairs: PF rank-one terms per covering output node a of an
    // expansion level-bank that has an active pair, rows phi_f(site - a T)
    // (images summed), columns R_a[f][site]. The covering nodes and their
    // flags are read in parallel first.
    if (active_pairs(tv) > 0) {
        __shared__ int pnode[MAX_PAIR_LB * 5]; // (l << 16 | a) of flagged nodes, else -1
        // Covering output nodes per expansion level-bank (one thread each),
        // prefix by warp 0, then one node per entry.
        static_assert(2 * MAX_PAIR_LB + 1 <= WT_THREADS && MAX_PAIR_LB <= 32,
                      "level-bank firsts and prefix fit ccls; one bank per lane");
        int *lfirst = ccls, *lpre = ccls + MAX_PAIR_LB; // ccls is free again
        if (t < g.npl) {
            int fo = 0, co = 0;
            if (g.pl_exp[t])
                co = cover_nodes(R0, TR, g.pl_T[t], g.pl_K[t] * g.pl_T[t], g.pl_no[t], no, fo);
            lfirst[t] = fo;
            lpre[t + 1] = co;
        }
        __syncthreads();
        if (warp == 0) {
            int inc = lane < g.npl ? lpre[lane + 1] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            if (lane < g.npl) lpre[lane + 1] = inc;
            if (lane == 0) lpre[0] = 0;
        }
        __syncthreads();
        const int np = lpre[g.npl];
        for (int i = t; i < np; i += WT_THREADS) {
            int lo = 0, hi = g.npl - 1; // last bank with lpre[l] <= i
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (lpre[mid] <= i) lo = mid;
                else hi = mid - 1;
            }
            const int l = lo, rem = i - lpre[l], fo = lfirst[l];
            const int a = fo + rem >= g.pl_no[l] ? fo + rem - g.pl_no[l] : fo + rem;
            pnode[i] = tv.node_on[g.pl_node[l] + a] ? (l << 16 | a) : -1;
        }
        __syncthreads();
        // Up to three flagged nodes per pass (3 PF <= WT_STAGE staged terms):
        // warp k stages the rows of node k, every thread the columns.
        constexpr int PER_PASS = WT_STAGE / PF;
        int i = 0;
        while (true) {
            int key[PER_PASS], nn = 0;
            for (; i < np && nn < PER_PASS; ++i)
                if (pnode[i] >= 0) key[nn++] = pnode[i]; // CTA-uniform
            if (nn == 0) break;
            // Terms k PF + f: rows phi_f of node k (warp k, lane = tile row),
            // columns R_a[f] (every thread); columns up to the MMA's multiple
            // of 8 are zero.
            const int nt = nn * PF, kpad = (nt + 7) & ~7;
            if (warp < nn) {
                const int l = key[warp] >> 16, a = key[warp] & 0xFFFF;
                const int T = g.pl_T[l], F = g.pl_K[l] * T;
                float phi[PF];
                const bool on = lane < TR && pair_basis(R0 + lane - a * T, F, no, phi);
#pragma unroll
                for (int f = 0; f < PF; ++f) us[lane][warp * PF + f] = on ? phi[f] : 0.f;
            }
            for (int e = t; e < nt * TS; e += WT_THREADS) {
                const int k = e / (PF * TS), rem = e - k * (PF * TS);
                const int f = rem / TS, c = rem - f * TS;
                const int l = key[k] >> 16, a = key[k] & 0xFFFF;
                const float *rb = tv.pair_buf + g.pl_buf[l] + ((long long)a * PF + f) * ni + C0;
                vs[c][k * PF + f] = c < TC ? rb[c] : 0.f;
            }
            for (int e = t; e < 2 * TS * (kpad - nt); e += WT_THREADS) {
                const int pl = e >= TS * (kpad - nt), rem = e - pl * TS * (kpad - nt);
                const int r = rem / (kpad - nt), k = nt + rem - r * (kpad - nt);
                (pl ? vs : us)[r][k] = 0.f;
            }
            __syncthreads();
            tile_mma(acc, us, vs, kpad, warp, lane);
            __syncthreads();
        }
    }

    // Accumulator of warp w, n-tile nt: rows 16 (w / 2) + g (+8), columns
    // 16 (w % 2) + 8 nt + 2q (+1).
    float vmax = 0.f;
    {
        const int g = lane >> 2, q = lane & 3;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = (warp >> 1) * 16 + g + (e >= 2 ? 8 : 0);
                const int c = (warp & 1) * 16 + nt * 8 + 2 * q + (e & 1);
                if (r >= TR || c >= TC) continue;
                const long long row = R0 - out.r0 + r, col = C0 - out.c0 + c;
                const float v = acc[nt][e];
                vmax = fmaxf(vmax, fabsf(v));
                if (out.w) out.w[row * out.ldw + col] = v;
                if (out.hi) {
                    const float h = tf32_rna(v);
                    out.hi[row * out.lds + col] = h;
                    out.lo[row * out.lds + col] = tf32_rna(v - h);
                }
            }
    }
    if (out.amax) block_max_to(out.amax, vmax);
}

__global__ void split_kernel(const float *__restrict__ x, int cols, long long ldx,
                             float *__restrict__ hi, float *__restrict__ lo, long long ldo) {
    pdl_wait();
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
    pdl_wait();
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

// max |x| over a [rows][cols] view into *amax (which must start at 0 or lower).
// Blocks take four rows at a time (four independent loads in flight per
// thread), threads the row's float4s (or floats).
constexpr int ROWS_PER_PASS = 4;

__global__ void __launch_bounds__(256) absmax_kernel(const float *__restrict__ x, long long rows,
                                                     int cols, long long ld, int vec,
                                                     float *__restrict__ amax) {
    pdl_wait();
    float m = 0.f;
    const int n = vec ? cols / 4 : cols;
    for (long long r0 = blockIdx.x * (long long)ROWS_PER_PASS; r0 < rows;
         r0 += (long long)gridDim.x * ROWS_PER_PASS) {
        for (int c = threadIdx.x; c < n; c += blockDim.x) {
            if (vec) {
                float4 v[ROWS_PER_PASS];
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u)
                    v[u] = r0 + u < rows ? reinterpret_cast<const float4 *>(x + (r0 + u) * ld)[c]
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u)
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)),
                                       fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
            } else {
                float v[ROWS_PER_PASS];
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u)
                    v[u] = r0 + u < rows ? x[(r0 + u) * ld + c] : 0.f;
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u) m = fmaxf(m, fabsf(v[u]));
            }
        }
    }
    block_max_to(amax, m);
}

__device__ __forceinline__ void split2(float a0, float a1, __half2 &h, __half2 &l) {
    h = __float22half2_rn(make_float2(a0, a1));
    const float2 b = __half22float2(h);
    l = __float22half2_rn(make_float2(a0 - b.x, a1 - b.y));
}

// F16 split: hi = rn_f16(s x), lo = rn_f16(s x - hi); s from *amax. Block 0
// stores s for the GEMM epilogue. Four rows per pass, as absmax_kernel.
__global__ void __launch_bounds__(256) split_f16_kernel(const float *__restrict__ x,
                                                        long long rows, int cols, long long ldx,
                                                        int vec, const float *__restrict__ amax,
                                                        __half *__restrict__ hi,
                                                        __half *__restrict__ lo, long long ldo,
                                                        float *__restrict__ scale_out) {
    pdl_wait();
    const float s = f16_scale(*amax);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
    const int n = vec ? cols / 4 : cols;
    for (long long r0 = blockIdx.x * (long long)ROWS_PER_PASS; r0 < rows;
         r0 += (long long)gridDim.x * ROWS_PER_PASS) {
        for (int c = threadIdx.x; c < n; c += blockDim.x) {
            if (vec) {
                float4 v[ROWS_PER_PASS];
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u)
                    if (r0 + u < rows) v[u] = reinterpret_cast<const float4 *>(x + (r0 + u) * ldx)[c];
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u) {
                    if (r0 + u >= rows) continue;
                    __half2 h0, l0, h1, l1;
                    split2(v[u].x * s, v[u].y * s, h0, l0);
                    split2(v[u].z * s, v[u].w * s, h1, l1);
                    uint2 hp, lp;
                    hp.x = *reinterpret_cast<unsigned *>(&h0);
                    hp.y = *reinterpret_cast<unsigned *>(&h1);
                    lp.x = *reinterpret_cast<unsigned *>(&l0);
                    lp.y = *reinterpret_cast<unsigned *>(&l1);
                    reinterpret_cast<uint2 *>(hi + (r0 + u) * ldo)[c] = hp;
                    reinterpret_cast<uint2 *>(lo + (r0 + u) * ldo)[c] = lp;
                }
            } else {
#pragma unroll
                for (int u = 0; u < ROWS_PER_PASS; ++u) {
                    if (r0 + u >= rows) continue;
                    const float a = x[(r0 + u) * ldx + c] * s;
                    const __half h = __float2half_rn(a);
                    hi[(r0 + u) * ldo + c] = h;
                    lo[(r0 + u) * ldo + c] = __float2half_rn(a - __half2float(h));
                }
            }
        }
    }
}

// MSE upstream gradient in float32: dY = (Y - T) * scale (dY may overwrite Y),
// per-block sums of (Y - T)^2 in double (fixed tree) and max |dY| into *amax.
__global__ void __launch_bounds__(256) mse_f32_kernel(const float *y, const float *__restrict__ t,
                                                      long long rows, int cols, long long ld,
                                                      float scale, float *dy, long long ldo,
                                                      double *__restrict__ partial, int vec,
                                                      float *__restrict__ amax) {
    pdl_wait();
    __shared__ double red[256];
    double acc = 0;
    float m = 0.f;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        if (vec) {
            const float4 *yr = reinterpret_cast<const float4 *>(y + r * ld);
            const float4 *tr = reinterpret_cast<const float4 *>(t + r * ld);
            float4 *dr = reinterpret_cast<float4 *>(dy + r * ldo);
            for (int c = threadIdx.x; c < cols / 4; c += blockDim.x) {
                const float4 a = yr[c], b = tr[c];
                const float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
                acc += double(d0) * d0 + double(d1) * d1 + double(d2) * d2 + double(d3) * d3;
                const float4 g = make_float4(d0 * scale, d1 * scale, d2 * scale, d3 * scale);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(g.x), fabsf(g.y)), fmaxf(fabsf(g.z), fabsf(g.w))));
                dr[c] = g;
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += blockDim.x) {
                const float d = y[r * ld + c] - t[r * ld + c];
                acc += double(d) * double(d);
                const float g = d * scale;
                m = fmaxf(m, fabsf(g));
                dy[r * ldo + c] = g;
            }
        }
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s2 = 128; s2 > 0; s2 >>= 1) {
        if (threadIdx.x < s2) red[threadIdx.x] += red[threadIdx.x + s2];
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
    if (amax) block_max_to(amax, m);
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
    pdl_wait();
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
    return std::max<int64_t>(cache_floats(atoms) * 4, 16);
}

static int assemble(const void *atom_table_dev, int64_t atoms, const AxisCfg &oa,
                    const AxisCfg &ia, void *scratch, float *weight_dev, int64_t ld_weight,
                    float *weight_hi_dev, float *weight_lo_dev, int64_t ld_split,
                    cudaStream_t st, float *amax_dev = nullptr,
                    Window win = Window{0, 0, -1, -1}) {
    if (win.wr < 0) win = Window{0, 0, oa.sites, ia.sites};
    if (reinterpret_cast<uintptr_t>(atom_table_dev) % 16) {
        tcst_set_error("weight assembly: the atom table must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    const int words = record_words(oa.modes, ia.modes);
    const Table tv = table_view(atom_table_dev, atoms, words, axis_geo(oa), axis_geo(ia));
    float *cache = static_cast<float *>(scratch);
    if (max_scan_entries(tv.geom, oa.sites, ia.sites) > MAX_SCAN) {
        tcst_set_error("weight assembly: a weight tile would scan more than %d bins", MAX_SCAN);
        return TCST_ERR_UNSUPPORTED;
    }
    int rc = 0;
    {
        // The mass cache and the owner-pair coefficients and expansions are
        // independent: the pair kernels run on a side stream, joined before
        // the gather.
        SideStreams side(st, 1);
        if ((rc = side.status())) return rc;
        if (atoms > 0 && tv.geom.nclass > 0) {
            // The class range is only known on the device; the kernel reads it.
            const long long warps = std::min<long long>(atoms, sm_count() * 64LL);
            const cudaError_t e = launch_pdl(mass_cache_kernel, dim3(unsigned((warps + 7) / 8)),
                                             dim3(256), 0, st, tv, cache);
            if (e != cudaSuccess) rc = tcst_cuda_check(e, "mass_cache_kernel");
        }
        if (!rc) rc = pair_forward(tv, oa, ia, win, side[0]);
        const int rj = side.join();
        if (rc || (rc = rj)) return rc;
    }
    if (win.wr == 0 || win.wc == 0) return TCST_OK;
    const int tiles_r = (win.wr + TS - 1) / TS, tiles_c = (win.wc + TS - 1) / TS;
    GatherOut out = {weight_dev, weight_hi_dev, weight_lo_dev, ld_weight, ld_split, amax_dev,
                     win.r0, win.c0, win.wr, win.wc};
    TCST_CUDA(launch_pdl(weight_gather_kernel, dim3(unsigned(tiles_r * tiles_c)), dim3(WT_THREADS), 0, st, 
        tv, oa.sites, ia.sites, oa.modes, ia.modes, tiles_c, cache, out));
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
        scratch_bytes < cache_floats(atoms) * 4 ||
        reinterpret_cast<uintptr_t>(scratch_dev) % 16 ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    return assemble(atom_table_dev, atoms, oa, ia, scratch_dev, weight_dev, ld_weight,
                    weight_hi_dev, weight_lo_dev, ld_split, (cudaStream_t)stream);
}

static int assemble_f16(const char *name, const void *atom_table_dev, int64_t atoms,
                        const tcst_axis *out_axis, const tcst_axis *in_axis, void *scratch_dev,
                        int64_t scratch_bytes, int64_t r0, int64_t wr, int64_t c0, int64_t wc,
                        float *weight_dev, int64_t ld_weight, float *amax_dev, void *hi_dev,
                        void *lo_dev, int64_t ld_split, float *scale_dev, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (wr < 0) r0 = 0, wr = oa.sites;
    if (wc < 0) c0 = 0, wc = ia.sites;
    if (atoms < 0 || !scratch_dev || !atom_table_dev || !weight_dev || !amax_dev || !hi_dev ||
        !lo_dev || !scale_dev || scratch_bytes < cache_floats(atoms) * 4 ||
        reinterpret_cast<uintptr_t>(scratch_dev) % 16 || ld_weight < wc || ld_split < wc ||
        r0 < 0 || c0 < 0 || r0 + wr > oa.sites || c0 + wc > ia.sites || r0 % TS || c0 % TS) {
        tcst_set_error("%s: invalid arguments", name);
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if ((rc = assemble(atom_table_dev, atoms, oa, ia, scratch_dev, weight_dev, ld_weight, nullptr,
                       nullptr, 0, st, amax_dev, Window{int(r0), int(c0), int(wr), int(wc)})))
        return rc;
    return tcst_split_f16(weight_dev, wr, wc, ld_weight, amax_dev, hi_dev, lo_dev, ld_split,
                          scale_dev, stream);
}

extern "C" int tcst_assemble_weight_f16(const void *atom_table_dev, int64_t atoms,
                                        const tcst_axis *out_axis, const tcst_axis *in_axis,
                                        void *scratch_dev, int64_t scratch_bytes,
                                        float *weight_dev, int64_t ld_weight, float *amax_dev,
                                        void *hi_dev, void *lo_dev, int64_t ld_split,
                                        float *scale_dev, void *stream) {
    return assemble_f16("tcst_assemble_weight_f16", atom_table_dev, atoms, out_axis, in_axis,
                        scratch_dev, scratch_bytes, 0, -1, 0, -1, weight_dev, ld_weight, amax_dev,
                        hi_dev, lo_dev, ld_split, scale_dev, stream);
}

extern "C" int tcst_assemble_weight_window_f16(const void *atom_table_dev, int64_t atoms,
                                               const tcst_axis *out_axis,
                                               const tcst_axis *in_axis, void *scratch_dev,
                                               int64_t scratch_bytes, int64_t row0, int64_t rows,
                                               int64_t col0, int64_t cols, float *weight_dev,
                                               int64_t ld_weight, float *amax_dev, void *hi_dev,
                                               void *lo_dev, int64_t ld_split, float *scale_dev,
                                               void *stream) {
    if (rows < 0 || cols < 0) {
        tcst_set_error("tcst_assemble_weight_window_f16: negative window");
        return TCST_ERR_ARGUMENT;
    }
    return assemble_f16("tcst_assemble_weight_window_f16", atom_table_dev, atoms, out_axis,
                        in_axis, scratch_dev, scratch_bytes, row0, rows, col0, cols, weight_dev,
                        ld_weight, amax_dev, hi_dev, lo_dev, ld_split, scale_dev, stream);
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
        TCST_CUDA(launch_pdl(split4_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, st, 
            (const float4 *)x_dev, rows, int(cols / 4), ld_x / 4, (float4 *)hi_dev,
            (float4 *)lo_dev, ld_out / 4));
    } else {
        if (rows > 65535) {
            tcst_set_error("tcst_split_tf32: unaligned rows limited to 65535");
            return TCST_ERR_UNSUPPORTED;
        }
        dim3 grid(unsigned((cols + 255) / 256), unsigned(rows));
        TCST_CUDA(launch_pdl(split_kernel, dim3(grid), dim3(256), 0, st, x_dev, int(cols), ld_x, hi_dev, lo_dev, ld_out));
    }
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_absmax(const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                           float *amax_dev, void *stream) {
    if (rows < 0 || cols < 0 || !amax_dev || (rows * cols && (!x_dev || ld < cols))) {
        tcst_set_error("tcst_absmax: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if (rows * cols == 0) return TCST_OK;
    const int vec = cols % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(x_dev) & 15) == 0;
    const long long blocks =
        std::min<long long>((rows + ROWS_PER_PASS - 1) / ROWS_PER_PASS, sm_count() * 8LL);
    TCST_CUDA(launch_pdl(absmax_kernel, dim3(unsigned(blocks)), dim3(256), 0, (cudaStream_t)stream, x_dev, rows, int(cols), ld,
                                                                       vec, amax_dev));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_split_f16(const float *x_dev, int64_t rows, int64_t cols, int64_t ld_x,
                              const float *amax_dev, void *hi_dev, void *lo_dev, int64_t ld_out,
                              float *scale_dev, void *stream) {
    if (rows < 0 || cols < 0 || !amax_dev || !scale_dev) {
        tcst_set_error("tcst_split_f16: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if (rows * cols == 0) return TCST_OK;
    if (ld_x < cols || ld_out < cols || !x_dev || !hi_dev || !lo_dev) {
        tcst_set_error("tcst_split_f16: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    const int vec = cols % 4 == 0 && ld_x % 4 == 0 && ld_out % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(x_dev) & 15) |
                     (reinterpret_cast<uintptr_t>(hi_dev) & 7) |
                     (reinterpret_cast<uintptr_t>(lo_dev) & 7)) == 0;
    const long long blocks =
        std::min<long long>((rows + ROWS_PER_PASS - 1) / ROWS_PER_PASS, sm_count() * 8LL);
    TCST_CUDA(launch_pdl(split_f16_kernel, dim3(unsigned(blocks)), dim3(256), 0, (cudaStream_t)stream, 
        x_dev, rows, int(cols), ld_x, vec, amax_dev, (__half *)hi_dev, (__half *)lo_dev, ld_out,
        scale_dev));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

extern "C" int tcst_mse_grad_f32(const float *y_dev, const float *target_dev, int64_t rows,
                                 int64_t cols, int64_t ld, float scale, float *dy_dev,
                                 int64_t ld_out, double *loss_partial_dev, int32_t *blocks,
                                 float *amax_dev, void *stream) {
    const int nblocks = sm_count() * 4;
    if (blocks) *blocks = nblocks;
    if (rows < 0 || cols < 1 || ld < cols || ld_out < cols || !loss_partial_dev ||
        (rows && (!y_dev || !target_dev || !dy_dev))) {
        tcst_set_error("tcst_mse_grad_f32: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    if (dy_dev == y_dev && ld_out != ld) {
        tcst_set_error("tcst_mse_grad_f32: dY may overwrite Y only with the same leading dimension");
        return TCST_ERR_ARGUMENT;
    }
    const int vec =
        cols % 4 == 0 && ld % 4 == 0 && ld_out % 4 == 0 &&
        ((reinterpret_cast<uintptr_t>(y_dev) | reinterpret_cast<uintptr_t>(target_dev) |
          reinterpret_cast<uintptr_t>(dy_dev)) % 16) == 0;
    TCST_CUDA(launch_pdl(mse_f32_kernel, dim3(nblocks), dim3(256), 0, (cudaStream_t)stream, y_dev, target_dev, rows, int(cols), ld,
                                                              scale, dy_dev, ld_out,
                                                              loss_partial_dev, vec, amax_dev));
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
    TCST_CUDA(launch_pdl(mse_kernel, dim3(nblocks), dim3(256), 0, (cudaStream_t)stream, y_dev, target_dev, rows, int(cols), ld,
                                                          scale, dy_hi_dev, dy_lo_dev, ld_out,
                                                          loss_partial_dev, vec));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

// ---------------------------------------------------------------------------
// Weight assembly without caller-provided scratch.
//
// Some callers cannot hand this library device memory for the assembly's
// scratch (the mass cache of mid-size footprints): a plugin running inside a
// host framework whose allocator owns every device byte, or a fixed-footprint
// deployment that forbids allocation after start-up. For them the scratch
// lives in a fixed array compiled into this library. Every GPU that loads the
// library holds the array until the process exits.
// ---------------------------------------------------------------------------

namespace {

constexpr long long STATIC_SCRATCH_BYTES = 32LL << 20; // 32 MiB: up to 32768 atoms
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) float g_static_scratch[STATIC_SCRATCH_BYTES / 4];

std::mutex g_static_mutex;
void *g_static_ptr[MAX_DEVICES] = {};

// Host code must not pass g_static_scratch itself to a kernel: in host code that
// name is only a stand-in. The device address comes from cudaGetSymbolAddress,
// taken once per device with that device current. The cache needs no
// initialization: every call writes the entries it reads.
int static_scratch(void **out) {
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
    if (atoms < 0) {
        tcst_set_error("tcst_assemble_weight_static: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    // Range first, so the byte count below cannot overflow: the scratch holds
    // 2 x CACHE_SITES floats per atom.
    if (atoms > STATIC_SCRATCH_BYTES / (8LL * CACHE_SITES) ||
        cache_floats(atoms) * 4 > STATIC_SCRATCH_BYTES) {
        tcst_set_error("tcst_assemble_weight_static: %lld atoms need more than the built-in "
                       "%lld scratch bytes (%lld atoms at most); use tcst_assemble_weight",
                       (long long)atoms, STATIC_SCRATCH_BYTES,
                       STATIC_SCRATCH_BYTES / (8LL * CACHE_SITES));
        return TCST_ERR_UNSUPPORTED;
    }
    if (!atom_table_dev ||
        ((weight_hi_dev == nullptr) != (weight_lo_dev == nullptr)) ||
        (weight_dev && ld_weight < ia.sites) || (weight_hi_dev && ld_split < ia.sites)) {
        tcst_set_error("tcst_assemble_weight_static: invalid arguments");
        return TCST_ERR_ARGUMENT;
    }
    cudaStream_t st = (cudaStream_t)stream;
    void *scratch = nullptr;
    if ((rc = static_scratch(&scratch))) return rc;
    return assemble(atom_table_dev, atoms, oa, ia, scratch, weight_dev, ld_weight, weight_hi_dev,
                    weight_lo_dev, ld_split, st);
}
