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

__host__ __device__ inline int axis_words(int modes) { return 4 + 2 * (modes + 1); }
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
    double h = ddiv(ax.spacing, 2.0);
    double v = dsub(ddiv(dadd(r.local, h), width), ddiv(double(r.count - 1), 2.0));
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

__host__ int make_axis(const tcst_axis *in, AxisCfg *out, char *err, int errlen);
__host__ int make_coords(const tcst_coordinates *in, const AxisCfg &out_ax,
                         const AxisCfg &in_ax, CoordCfg *out, char *err, int errlen);

} // namespace tcst

// Host-side error reporting shared by all entry points.
void tcst_set_error(const char *fmt, ...);
int tcst_cuda_check(cudaError_t e, const char *what);

#define TCST_CUDA(call)                                                          \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) return tcst_cuda_check(e_, #call);                \
    } while (0)
