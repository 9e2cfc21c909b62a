// Shared device code of the B200 cell-mass Linear backend.
//
// Atom record (one per atom, RECORD_WORDS 32-bit words, 16-byte aligned):
//   word 0  amp     float32  physical amplitude (rational: a; Polar: amax*s/|(s,t)|)
//   word 1  chain0  float32  dr/da (rational) or d amp/ds (Polar)
//   word 2  chain1  float32  dr/dq (rational) or d amp/dt (Polar)
//   word 3  flags   int32    bit0 Polar (radius detached), bit1 invalid atom
//   then one axis block per axis, output axis first:
//     +0 first   int32   first unwrapped site = first_tile * tile_sites
//     +1 length  int32   footprint length F = K * tile_sites (one local period)
//     +2 phase0  float32 2 (first*s - mu_rel) / P, in half turns
//     +3 omega   float32 2 pi / P
//     +4 .. +4+M          coef_k  = s c_k sinc(k s/P) (x2 for k >= 1)
//     +5+M .. +5+2M       dcoef_k = d coef_k / dR
// A footprint site j (0 <= j < F) sits at chart site (first + j) mod N and has
// half-turn phase t_j = phase0 + 2 j / F, so
//   m(j)      = sum_k coef_k  cos(pi k t_j)
//   dm/dR(j)  = sum_k dcoef_k cos(pi k t_j)
//   dm/dmu(j) = omega * sum_k k coef_k sin(pi k t_j).
#pragma once

#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "../../include/tcst_b200.h"

namespace tcst {

constexpr int MAX_MODES = 16;
constexpr int MAX_LEVELS = 31;
constexpr double PI = 3.14159265358979323846;

struct AxisCfg {
    int sites, base, merge, modes, levels;
    double spacing, origin, period;
    int node_offset[2 * MAX_LEVELS]; // per bank (level*2 + K-2)
    int node_count;
};

struct CoordCfg {
    int kind;
    double amax;
    double rmin, rbirth, rmax;
    float lo32, hi32; // representable clamp interval of the rational radius
    double w_c, kappa, lower_kappa, udp;
    double ob[4], ib[4];
};

// Axis blocks are padded to 16 bytes so both start aligned and store as float4s.
__host__ __device__ inline int axis_words(int modes) { return (4 + 2 * (modes + 1) + 3) & ~3; }
__host__ __device__ inline int record_words(int modes_out, int modes_in) {
    int w = 4 + axis_words(modes_out) + axis_words(modes_in);
    return (w + 3) & ~3;
}

__device__ inline int wrap_site(long long s, int n) {
    long long r = s % n;
    return int(r < 0 ? r + n : r);
}

// Non-contracted double arithmetic: the reference evaluates each operation as a
// separate correctly rounded step, which routing must reproduce bit for bit.
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double ddiv(double a, double b) { return __ddiv_rn(a, b); }

struct Route {
    int level, count, tile, first_tile;
    double local; // relative center in [0, Q]
};

// _backends/torch/kernels/radius_cell_mass.py:17-63 (finite-period branch).
__device__ inline double relative_center(double mu, const AxisCfg &ax) {
    double residue = fmod(mu, ax.period);
    double origin_residue = fmod(ax.origin, ax.period);
    double rel = fmod(dsub(residue, origin_residue), ax.period);
    return rel < 0 ? dadd(rel, ax.period) : rel;
}

// _backends/torch/kernels/radius_cell_mass.py:84-104.
__device__ inline Route route_axis(double R, double mu, const AxisCfg &ax) {
    Route r;
    int tile = ax.base;
    int level = 0;
    for (; level < ax.levels - 1; ++level, tile *= ax.merge) {
        if (R <= dmul(double(tile), ax.spacing)) break;
    }
    double width = dmul(double(tile), ax.spacing);
    r.level = level;
    r.tile = tile;
    r.count = int(ceil(ddiv(dmul(2.0, R), width))) + 1;
    r.local = relative_center(mu, ax);
    // Halving by a product with 0.5: the same IEEE result as the division.
    double h = dmul(ax.spacing, 0.5);
    double v = dsub(ddiv(dadd(r.local, h), width), dmul(double(r.count - 1), 0.5));
    r.first_tile = int(floor(v));
    return r;
}

// Values of one footprint site from an axis block: m, dm/dR, dm/dmu.
struct SiteVals {
    float m, dR, dmu;
};

__device__ __forceinline__ float site_mass(const float *blk, int modes, int j, int F) {
    float t = blk[2] + 2.0f * float(j) / float(F);
    float s1, c1;
    sincospif(t, &s1, &c1);
    const float *coef = blk + 4;
    float acc = coef[0];
    float cprev = 1.0f, ccur = c1;
    for (int k = 1; k <= modes; ++k) {
        acc = fmaf(coef[k], ccur, acc);
        float cn = fmaf(2.0f * c1, ccur, -cprev);
        cprev = ccur;
        ccur = cn;
    }
    return acc;
}

__device__ __forceinline__ SiteVals site_values(const float *blk, int modes, int j, int F) {
    float t = blk[2] + 2.0f * float(j) / float(F);
    float s1, c1;
    sincospif(t, &s1, &c1);
    const float *coef = blk + 4;
    const float *dcoef = blk + 5 + modes;
    float m = coef[0], dR = dcoef[0], dmu = 0.0f;
    float cprev = 1.0f, ccur = c1, sprev = 0.0f, scur = s1;
    for (int k = 1; k <= modes; ++k) {
        m = fmaf(coef[k], ccur, m);
        dR = fmaf(dcoef[k], ccur, dR);
        dmu = fmaf(float(k) * coef[k], scur, dmu);
        float cn = fmaf(2.0f * c1, ccur, -cprev);
        float sn = fmaf(2.0f * c1, scur, -sprev);
        cprev = ccur;
        ccur = cn;
        sprev = scur;
        scur = sn;
    }
    return {m, dR, dmu * blk[3]};
}

// ---------------------------------------------------------------------------
// Atom table layout (one buffer per decode call, saved for the backward pass):
//   records [atoms][words]
//   spans   [atoms] int4: output first site wrapped, output footprint,
//                         input first site wrapped, input footprint
//   sites   [atoms][2 axes][3 values][REACH]: m, dm/dmu, dm/dR of the first
//           REACH footprint sites of each axis (filled when F <= REACH, i.e.
//           for the site classes 0 .. SITE_CLASSES-1)
//   bin_of  [atoms] int: the atom's bin
//   offsets [nbins + 1] int, ids [atoms] int: atom ids grouped by bin, in
//           increasing id order inside every bin (stable counting sort)
//   counts  [sort_blocks + 1][nbins] int: sort workspace
//   sync    one word (+ padding): finished blocks of the sort's column prefix
//
// Bins. An atom's class is the smallest c whose reach class_reach(c) covers
// its larger footprint max(F_out, F_in), reach 16 << c. Classes 0..NFINE-1
// (reach 16, 32, 64, 128) are binned by the fe x fe tile of (output first
// site, input first site),
// fe = TS (2 TS for charts so large that TS bins do not fit);
// coarser classes (reach 256, 512, ... up to twice the larger axis, the widest
// footprint routing produces) by tiles of edge reach / 2. Bins are numbered
// class by class, tiles row-major, and invalid atoms take the last bin. When
// the geometry is not binned (mode counts other than 8, or more bins than the
// sort handles) every valid atom is in class-free bin 0.
//
// Owner pairs. When both axes share the tile hierarchy (base, merge, spacing),
// a coarse atom whose level and bank (tile T, count K) agree on both axes is
// binned by its owner pair (T, K, first tile out, first tile in) instead: one
// "pair level-bank" per (T, K) with K T > 128 and at most PAIR_BIN_CAP pairs,
// pair bins numbered after the class bins. All atoms of a pair share the
// footprint, so with the 2M+1 = PF functions phi_f(j) = {1, cos 2 pi k j/F,
// sin 2 pi k j/F} of the footprint site j, m_a(j) = sum_f alpha_a,f phi_f(j)
// and the pair's W block is Phi_out C Phi_in^T with
// C = sum_a amp_a alpha_out,a alpha_in,a^T (PF x PF). A pair with at least
// PAIR_MIN atoms in a level-bank that has an expansion buffer ("active") takes
// that path in the weight assembly and the pullback; the atoms of other pairs
// are treated one by one like any coarse atom.
// ---------------------------------------------------------------------------
constexpr int REACH = 32;        // footprint sites whose values the decode stores
constexpr int SITE_CLASSES = 2;  // classes with footprints of at most REACH sites
constexpr int SITE_FLOATS = 2 * 3 * REACH;
constexpr int TS = 32;          // fine bin tile edge and weight tile edge, in sites
constexpr int NFINE = 4;        // classes binned by TS tiles
constexpr int MAX_CLASSES = 16;
constexpr int MAX_BINS = 98304;  // 16-bit per-CTA bin counters fit in shared memory
constexpr int SORT_CHUNK = 512;  // atoms per sort block (128 blocks, more for > 8M atoms)
constexpr int CACHE_SITES = 128; // masses cached per axis for classes SITE_CLASSES..NFINE-1
constexpr int PF = 17;                // owner-pair basis functions per axis (M = 8)
constexpr int MAX_PAIR_LB = 32;       // pair level-banks
constexpr int PAIR_MIN = 2;           // atoms that make an owner pair active
constexpr int PAIR_BIN_CAP = 16384;   // owner pairs of a level-bank binned as pairs
constexpr int PAIR_EXPAND_CAP = 16384; // owner pairs of a level-bank with an expansion buffer

// What the bin geometry needs of an axis.
struct AxisGeo {
    int sites, base, merge, modes;
    double spacing;
};

__host__ __device__ constexpr int class_reach(int c) { return 16 << c; }
static_assert(class_reach(SITE_CLASSES - 1) == REACH, "site classes end at REACH");
static_assert(class_reach(NFINE - 1) <= CACHE_SITES, "cached classes fit the mass cache");
// Bin edge of class c: fe (the geometry's fine edge, TS or 2 TS) for the fine
// classes, half the reach for coarser ones.
__host__ __device__ constexpr int class_edge(int c, int fe) {
    return c < NFINE ? fe : class_reach(c) / 2;
}

__host__ __device__ inline long long align16(long long x) { return (x + 15) & ~15LL; }

struct BinGeom {
    int nclass;                   // 0 when not binned
    int fe;                       // fine bin edge (TS, or 2 TS when TS bins do not fit)
    int tr[MAX_CLASSES], tc[MAX_CLASSES]; // tiles per axis of each class
    int base[MAX_CLASSES + 1];    // first bin of each class; base[nclass] = first bin past them
    int nbins;                    // last pair bin + 2 (invalid bin)
    int sort_blocks;              // counting-sort blocks
    long long chunk;              // atoms per sort block
    // Owner-pair level-banks (npl = 0 without a shared hierarchy).
    int npl;
    int pl_T[MAX_PAIR_LB], pl_K[MAX_PAIR_LB];   // tile and count
    int pl_no[MAX_PAIR_LB], pl_ni[MAX_PAIR_LB]; // first tiles per axis (N / T)
    int pl_base[MAX_PAIR_LB + 1];               // first bin; pl_base[npl] = invalid bin
    int pl_exp[MAX_PAIR_LB];                    // has an expansion buffer
    int pl_node[MAX_PAIR_LB];                   // first node flag of the level-bank
    long long pl_buf[MAX_PAIR_LB];              // float offset of its [no][PF][N_in] buffer
    int pl_of[2 * MAX_LEVELS];                  // level * 2 + K - 2 -> level-bank or -1
    int nodes;                                  // node flags
    long long buf_floats;                       // expansion buffer floats
};

__host__ __device__ inline BinGeom bin_geom(long long atoms, const AxisGeo &ao,
                                            const AxisGeo &ai) {
    BinGeom g;
    const int n_out = ao.sites, n_in = ai.sites, modes_out = ao.modes, modes_in = ai.modes;
    const int nmax = n_out > n_in ? n_out : n_in;
    int nc = 0;
    long long nb = 0;
    // Fine bins of TS sites per side, or of 2 TS when those do not fit.
    for (g.fe = TS; g.fe <= 2 * TS; g.fe *= 2) {
        nc = 0;
        nb = 0;
        while (nc < MAX_CLASSES) {
            const int e = class_edge(nc, g.fe);
            g.tr[nc] = (n_out + e - 1) / e;
            g.tc[nc] = (n_in + e - 1) / e;
            g.base[nc] = int(nb < 0x7fffffff ? nb : 0x7fffffff);
            nb += (long long)g.tr[nc] * g.tc[nc];
            ++nc;
            if (class_reach(nc - 1) >= 2 * nmax) break;
        }
        if (nb + 1 <= MAX_BINS) break;
    }
    if (g.fe > 2 * TS) g.fe = 2 * TS;
    const long long class_end = nb;
    g.npl = 0;
    g.nodes = 0;
    g.buf_floats = 0;
    for (int i = 0; i < 2 * MAX_LEVELS; ++i) g.pl_of[i] = -1;
    const bool binned =
        modes_out == 8 && modes_in == 8 && nb + 1 <= MAX_BINS && class_reach(nc - 1) >= 2 * nmax;
    if (binned && ao.base == ai.base && ao.merge == ai.merge && ao.spacing == ai.spacing &&
        ao.merge > 1 && ao.base > 0) {
        long long t = ao.base;
        for (int level = 0; level < MAX_LEVELS && t <= n_out && t <= n_in; ++level) {
            for (int k = 2; k <= 3 && g.npl < MAX_PAIR_LB; ++k) {
                const long long no = n_out / t, ni = n_in / t;
                if (k * t <= class_reach(NFINE - 1) || no * ni > PAIR_BIN_CAP ||
                    n_out % t || n_in % t || nb + no * ni + 1 > MAX_BINS)
                    continue;
                const int l = g.npl++;
                g.pl_T[l] = int(t);
                g.pl_K[l] = k;
                g.pl_no[l] = int(no);
                g.pl_ni[l] = int(ni);
                g.pl_base[l] = int(nb);
                g.pl_exp[l] = no * ni <= PAIR_EXPAND_CAP;
                g.pl_node[l] = g.nodes;
                g.pl_buf[l] = g.buf_floats;
                if (g.pl_exp[l]) {
                    g.nodes += int(no);
                    g.buf_floats += no * PF * n_in;
                }
                g.pl_of[2 * level + k - 2] = l;
                nb += no * ni;
            }
            t *= ao.merge;
        }
    }
    g.pl_base[g.npl] = int(nb);
    if (!binned) {
        g.nclass = 0;
        g.npl = 0;
        g.pl_base[0] = 1;
        g.base[0] = 0;
        g.nbins = 2; // bin 0: every valid atom; bin 1: invalid atoms
    } else {
        g.nclass = nc;
        g.base[nc] = int(class_end);
        g.nbins = int(nb) + 1;
    }
    // At most 128 blocks, but never more than 65,535 atoms per block (16-bit counters).
    long long blocks = (atoms + SORT_CHUNK - 1) / SORT_CHUNK;
    const long long at_least = (atoms + 65534) / 65535;
    blocks = blocks > 128 ? 128 : blocks;
    blocks = blocks < at_least ? at_least : blocks;
    blocks = blocks < 1 ? 1 : blocks;
    g.sort_blocks = int(blocks);
    g.chunk = (atoms + blocks - 1) / blocks;
    return g;
}

struct TableLayout {
    long long spans_off, sites_off, binof_off, offsets_off, ids_off, counts_off, sync_off,
        pair_c_off, node_off, buf_off, sspan_off, samp_off, total; // bytes
    BinGeom geom;
};

__host__ __device__ inline TableLayout table_layout(long long atoms, int words, const AxisGeo &ao,
                                                   const AxisGeo &ai) {
    TableLayout t;
    t.geom = bin_geom(atoms, ao, ai);
    t.spans_off = align16(atoms * words * 4);
    t.sites_off = align16(t.spans_off + atoms * 16);
    t.binof_off = align16(t.sites_off + atoms * SITE_FLOATS * 4);
    t.offsets_off = align16(t.binof_off + atoms * 4);
    t.ids_off = align16(t.offsets_off + 4LL * (t.geom.nbins + 1));
    t.counts_off = align16(t.ids_off + atoms * 4);
    t.sync_off = align16(t.counts_off + 4LL * t.geom.nbins * (t.geom.sort_blocks + 1));
    // Owner-pair region: C per pair bin, node flags, expansion buffers.
    const long long pair_bins = t.geom.npl ? t.geom.pl_base[t.geom.npl] - t.geom.pl_base[0] : 0;
    t.pair_c_off = t.sync_off + 16;
    t.node_off = align16(t.pair_c_off + 4LL * PF * PF * pair_bins);
    t.buf_off = align16(t.node_off + 4LL * t.geom.nodes);
    // Spans and amplitudes in sorted (ids) order, written by the scatter.
    t.sspan_off = align16(t.buf_off + 4LL * t.geom.buf_floats);
    t.samp_off = align16(t.sspan_off + atoms * 16);
    t.total = align16(t.samp_off + atoms * 4);
    return t;
}

// Device pointers into one atom table.
struct Table {
    const float *rec;
    int words;
    long long atoms;
    const int4 *spans;
    const float *sites;
    int *bin_of, *offsets, *ids, *counts;
    unsigned *sync; // [0] finished blocks of the column prefix (reset by the decode),
                    // [1] active owner pairs (written by the column prefix)
    float *pair_c;  // [pair bins][PF][PF]: C of active pairs
    int *node_on;   // [nodes]: output node has an active pair (expansion level-banks),
                    // written by the sort's column prefix
    float *pair_buf; // expansion buffers: R = C Phi_in^T summed per output node, then
                     // the pullback's projections P = Phi_out^T G
    int4 *sspan;     // spans[ids[k]] at sorted position k (scatter)
    float *samp;     // amplitude (record word 0) of ids[k] at sorted position k (scatter)
    BinGeom geom;
};

__host__ __device__ inline Table table_view(const void *base, long long atoms, int words,
                                            const AxisGeo &ao, const AxisGeo &ai) {
    const TableLayout l = table_layout(atoms, words, ao, ai);
    char *b = static_cast<char *>(const_cast<void *>(base));
    Table t;
    t.rec = reinterpret_cast<const float *>(b);
    t.words = words;
    t.atoms = atoms;
    t.spans = reinterpret_cast<const int4 *>(b + l.spans_off);
    t.sites = reinterpret_cast<const float *>(b + l.sites_off);
    t.bin_of = reinterpret_cast<int *>(b + l.binof_off);
    t.offsets = reinterpret_cast<int *>(b + l.offsets_off);
    t.ids = reinterpret_cast<int *>(b + l.ids_off);
    t.counts = reinterpret_cast<int *>(b + l.counts_off);
    t.sync = reinterpret_cast<unsigned *>(b + l.sync_off);
    t.pair_c = reinterpret_cast<float *>(b + l.pair_c_off);
    t.node_on = reinterpret_cast<int *>(b + l.node_off);
    t.pair_buf = reinterpret_cast<float *>(b + l.buf_off);
    t.sspan = reinterpret_cast<int4 *>(b + l.sspan_off);
    t.samp = reinterpret_cast<float *>(b + l.samp_off);
    t.geom = l.geom;
    return t;
}

// Level-bank of a pair bin (or -1).
__host__ __device__ inline int pair_lb(const BinGeom &g, int bin) {
    if (g.npl == 0 || bin < g.pl_base[0] || bin >= g.pl_base[g.npl]) return -1;
    int l = 0;
    while (bin >= g.pl_base[l + 1]) ++l;
    return l;
}

// Active owner pairs of the table (0: every pair kernel has nothing to do).
__device__ __forceinline__ unsigned active_pairs(const Table &tv) { return tv.sync[1]; }

// Whether a pair bin takes the owner-pair path.
__device__ __forceinline__ bool pair_active(const BinGeom &g, const int *offsets, int bin) {
    const int l = pair_lb(g, bin);
    return l >= 0 && g.pl_exp[l] && offsets[bin + 1] - offsets[bin] >= PAIR_MIN;
}

__host__ __device__ inline int atom_class(int4 span) {
    const int f = span.y > span.w ? span.y : span.w;
    int c = 0;
    while (class_reach(c) < f) ++c;
    return c;
}

// Bin of an atom from its spans and its (level, K) on both axes (invalid atoms
// have footprint 0).
__device__ __forceinline__ int atom_bin(int4 span, const BinGeom &g, int lvl_o, int k_o,
                                        int lvl_i, int k_i) {
    const int invalid = g.nbins - 1;
    if (span.y <= 0 || span.w <= 0) return invalid;
    if (g.nclass == 0) return 0;
    const int c = atom_class(span);
    if (c >= NFINE && lvl_o == lvl_i && k_o == k_i && lvl_o >= 0 && lvl_o < MAX_LEVELS) {
        const int l = g.pl_of[2 * lvl_o + k_o - 2];
        if (l >= 0) {
            const int t = g.pl_T[l];
            return g.pl_base[l] + (span.x / t) * g.pl_ni[l] + span.z / t;
        }
    }
    const int e = class_edge(c, g.fe);
    return g.base[c] + (span.x / e) * g.tc[c] + span.z / e;
}

// Per-axis profile of one atom held in registers (M known at compile time).
template <int M> struct AxisCoef {
    int first, F;
    float phase0, omega;
    float c[M + 1], dc[M + 1];
    // The axis block is read as float4s: records and their axis blocks are
    // multiples of 16 bytes in a 16-byte aligned table.
    __device__ __forceinline__ void load(const float *blk) {
        constexpr int NW = (6 + 2 * M + 3) / 4 * 4; // header + c + dc, padded
        float w[NW];
        const float4 *b4 = reinterpret_cast<const float4 *>(blk);
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
            const float4 v = b4[i];
            w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
        }
        first = __float_as_int(w[0]);
        F = __float_as_int(w[1]);
        phase0 = w[2];
        omega = w[3];
#pragma unroll
        for (int k = 0; k <= M; ++k) {
            c[k] = w[4 + k];
            dc[k] = w[5 + M + k];
        }
    }
    // Header and mass coefficients only (dcoef left unset).
    __device__ __forceinline__ void load_mass(const float *blk) {
        constexpr int NW = (5 + M + 3) / 4 * 4; // header + c, padded
        float w[NW];
        const float4 *b4 = reinterpret_cast<const float4 *>(blk);
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
            const float4 v = b4[i];
            w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
        }
        first = __float_as_int(w[0]);
        F = __float_as_int(w[1]);
        phase0 = w[2];
        omega = w[3];
#pragma unroll
        for (int k = 0; k <= M; ++k) c[k] = w[4 + k];
    }
    __device__ __forceinline__ float mass(int j) const {
        const float t = phase0 + 2.0f * float(j) / float(F);
        float s1, c1;
        sincospif(t, &s1, &c1);
        return mass_c(c1);
    }
    // Mass from c1 = cos(pi t).
    __device__ __forceinline__ float mass_c(float c1) const {
        float acc = c[0], cprev = 1.0f, ccur = c1;
#pragma unroll
        for (int k = 1; k <= M; ++k) {
            acc = fmaf(c[k], ccur, acc);
            const float cn = fmaf(2.0f * c1, ccur, -cprev);
            cprev = ccur;
            ccur = cn;
        }
        return acc;
    }
    __device__ __forceinline__ SiteVals values(int j) const {
        return values_at(phase0 + 2.0f * float(j) / float(F));
    }
    // Values at half-turn phase t.
    __device__ __forceinline__ SiteVals values_at(float t) const {
        float s1, c1;
        sincospif(t, &s1, &c1);
        return values_cs(c1, s1);
    }
    // Values from c1 = cos(pi t), s1 = sin(pi t).
    __device__ __forceinline__ SiteVals values_cs(float c1, float s1) const {
        float m = c[0], dR = dc[0], dmu = 0.0f;
        float cprev = 1.0f, ccur = c1, sprev = 0.0f, scur = s1;
#pragma unroll
        for (int k = 1; k <= M; ++k) {
            m = fmaf(c[k], ccur, m);
            dR = fmaf(dc[k], ccur, dR);
            dmu = fmaf(float(k) * c[k], scur, dmu);
            const float cn = fmaf(2.0f * c1, ccur, -cprev);
            const float sn = fmaf(2.0f * c1, scur, -sprev);
            cprev = ccur;
            ccur = cn;
            sprev = scur;
            scur = sn;
        }
        return {m, dR, dmu * omega};
    }
};

__host__ int make_axis(const tcst_axis *in, AxisCfg *out, char *err, int errlen);

__host__ __device__ inline AxisGeo axis_geo(const AxisCfg &a) {
    return AxisGeo{a.sites, a.base, a.merge, a.modes, a.spacing};
}
inline AxisGeo axis_geo(const tcst_axis &a) {
    return AxisGeo{a.site_count, a.base_tile_sites, a.merge_factor, a.modes, a.spacing};
}
__host__ int make_coords(const tcst_coordinates *in, const AxisCfg &out_ax,
                         const AxisCfg &in_ax, CoordCfg *out, char *err, int errlen);

} // namespace tcst

namespace tcst {

// Atom gradient from its four footprint sums (s_amp = sum G m_out m_in,
// s_mo / s_mi with dm/dmu on one axis, s_r = sum G (dm_out/dR m_in +
// m_out dm_in/dR)): the rational (a, q) chain (rational_radius.py:19-23), the
// amplitude chain only for Polar rows (radius detached), zero for invalid atoms.
__device__ __forceinline__ float4 atom_chain(const float *rec, float s_amp, float s_mo,
                                             float s_mi, float s_r) {
    const int flags = reinterpret_cast<const int *>(rec)[3];
    const float amp = rec[0], ch0 = rec[1], ch1 = rec[2];
    if (flags & 2) return make_float4(0.f, 0.f, 0.f, 0.f);
    if (flags & 1) return make_float4(s_amp * ch0, s_amp * ch1, amp * s_mo, amp * s_mi);
    const float d_r = amp * s_r;
    return make_float4(fmaf(d_r, ch0, s_amp), d_r * ch1, amp * s_mo, amp * s_mi);
}

// Programmatic dependent launch: every kernel of this library is launched with
// programmatic stream serialization, so its blocks may become resident while
// the previous kernel on the stream drains; each kernel calls pdl_wait() before
// it touches memory that a predecessor writes (griddepcontrol.wait returns
// once the predecessor grid has completed and its writes are visible).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

int launch_priority(cudaStream_t stream); // atoms.cu

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributePriority;
    attr[1].val.priority = launch_priority(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

} // namespace tcst

// Host-side error reporting shared by all entry points.
void tcst_set_error(const char *fmt, ...);
int tcst_cuda_check(cudaError_t e, const char *what);

#define TCST_CUDA(call)                                                          \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) return tcst_cuda_check(e_, #call);                \
    } while (0)

namespace tcst {

// Side streams for independent launches inside one entry point. The
// constructor makes n (<= MAX) side streams of the current device wait
// for the work queued so far on `st`; join() makes `st` wait for everything
// queued on them since. The streams are created once per device and shared, so
// the object holds the device's lock from fork to join (concurrent callers
// serialize their host-side launch sequences, not their device work). Under
// stream capture the side streams join the capture and are joined back before
// the entry point returns. The destructor joins if join() was not called.
class SideStreams {
  public:
    static constexpr int MAX = 4;
    SideStreams(cudaStream_t st, int n);
    ~SideStreams();
    SideStreams(const SideStreams &) = delete;
    SideStreams &operator=(const SideStreams &) = delete;
    int status() const { return rc_; }
    cudaStream_t operator[](int i) const { return side_[i]; }
    int join();

  private:
    cudaStream_t st_;
    cudaStream_t side_[MAX] = {};
    void *set_ = nullptr;
    int n_ = 0, rc_ = 0;
    bool joined_ = false;
};

} // namespace tcst
