// Per-atom decode, hierarchy routing and Chebyshev-square Fourier profile,
// then the bin sort and (beside it) the site values of narrow footprints.
//
// Two threads per atom (one per axis), float64 throughout. Routing (level, K,
// first tile, owner key) reproduces the reference's float64 operation order
// with non-contracted arithmetic, so it is bit-exact whenever exp/log agree in
// the last ulp.

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"

static thread_local char g_error[512] = "";

void tcst_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int tcst_cuda_check(cudaError_t e, const char *what) {
    tcst_set_error("CUDA error in %s: %s", what, cudaGetErrorString(e));
    return TCST_ERR_CUDA;
}

extern "C" const char *tcst_last_error(void) { return g_error; }
extern "C" const char *tcst_version(void) { return "tcst_b200 1.0 sm_100a"; }

namespace tcst {

namespace {
struct SideSet {
    std::mutex mu;
    std::atomic<bool> ready{false};
    cudaStream_t s[SideStreams::MAX];
    cudaEvent_t fork, join[SideStreams::MAX];
};
constexpr int MAX_SIDE_DEVICES = 64;
SideSet g_sides[MAX_SIDE_DEVICES];

cudaError_t create_side_set(SideSet &set, int dev) {
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess && cur != dev) e = cudaSetDevice(dev);
    for (int i = 0; e == cudaSuccess && i < SideStreams::MAX; ++i) {
        e = cudaStreamCreateWithFlags(&set.s[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&set.join[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&set.fork, cudaEventDisableTiming);
    if (cur != dev) {
        const cudaError_t e2 = cudaSetDevice(cur);
        if (e == cudaSuccess) e = e2;
    }
    return e;
}
} // namespace

// Launch priority: the library's side streams run at the device's least
// priority, every other stream (the caller's, which carries the step's
// dependent chain) at its greatest, so that when both have blocks waiting the
// chain's go first.
int launch_priority(cudaStream_t stream) {
    static int least = 0, greatest = 0;
    static std::once_flag once;
    std::call_once(once, [] {
        if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) {
            cudaGetLastError();
            least = greatest = 0;
        }
    });
    for (int d = 0; d < MAX_SIDE_DEVICES; ++d) {
        if (!g_sides[d].ready.load(std::memory_order_acquire)) continue;
        for (int i = 0; i < SideStreams::MAX; ++i)
            if (g_sides[d].s[i] == stream) return least;
    }
    return greatest;
}

SideStreams::SideStreams(cudaStream_t st, int n) : st_(st) {
    // The calling stream belongs to the current device (as for every launch
    // here); cudaStreamGetDevice is not permitted while the stream captures.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        rc_ = tcst_cuda_check(e, "cudaGetDevice");
        return;
    }
    if (dev < 0 || dev >= MAX_SIDE_DEVICES || n < 0 || n > MAX) {
        tcst_set_error("side streams: device %d or count %d out of range", dev, n);
        rc_ = TCST_ERR_UNSUPPORTED;
        return;
    }
    SideSet &set = g_sides[dev];
    set.mu.lock();
    set_ = &set;
    if (!set.ready.load(std::memory_order_acquire)) {
        if ((e = create_side_set(set, dev)) != cudaSuccess) {
            rc_ = tcst_cuda_check(e, "side stream creation");
            return;
        }
        set.ready.store(true, std::memory_order_release);
    }
    if ((e = cudaEventRecord(set.fork, st)) != cudaSuccess) {
        rc_ = tcst_cuda_check(e, "cudaEventRecord (fork)");
        return;
    }
    for (; n_ < n; ++n_) {
        if ((e = cudaStreamWaitEvent(set.s[n_], set.fork, 0)) != cudaSuccess) {
            rc_ = tcst_cuda_check(e, "cudaStreamWaitEvent (fork)");
            return;
        }
        side_[n_] = set.s[n_];
    }
}

int SideStreams::join() {
    if (!set_) return rc_;
    SideSet &set = *static_cast<SideSet *>(set_);
    int rc = rc_;
    for (int i = 0; i < n_; ++i) {
        cudaError_t e = cudaEventRecord(set.join[i], side_[i]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st_, set.join[i], 0);
        if (e != cudaSuccess && rc == 0) rc = tcst_cuda_check(e, "side stream join");
    }
    joined_ = true;
    set_ = nullptr;
    set.mu.unlock();
    return rc;
}

SideStreams::~SideStreams() {
    if (set_) join();
}

__host__ int make_axis(const tcst_axis *in, AxisCfg *out, char *err, int errlen) {
    if (!in) {
        snprintf(err, errlen, "axis declaration is NULL");
        return TCST_ERR_ARGUMENT;
    }
    if (in->site_count < 1 || in->base_tile_sites < 1 || in->merge_factor < 2 ||
        in->modes < 1 || !(in->spacing > 0) || !std::isfinite(in->spacing) ||
        !std::isfinite(in->origin)) {
        snprintf(err, errlen, "invalid axis declaration");
        return TCST_ERR_ARGUMENT;
    }
    if (in->modes > MAX_MODES) {
        snprintf(err, errlen, "Chebyshev modes %d exceed this build's limit %d", in->modes,
                 MAX_MODES);
        return TCST_ERR_UNSUPPORTED;
    }
    if (in->site_count % in->base_tile_sites) {
        snprintf(err, errlen, "base_tile_sites must divide the chart site count");
        return TCST_ERR_ARGUMENT;
    }
    int ratio = in->site_count / in->base_tile_sites;
    while (ratio > 1 && ratio % in->merge_factor == 0) ratio /= in->merge_factor;
    if (ratio != 1) {
        snprintf(err, errlen, "chart/base tile ratio must be a power of merge_factor");
        return TCST_ERR_ARGUMENT;
    }
    memset(out, 0, sizeof(*out));
    out->sites = in->site_count;
    out->base = in->base_tile_sites;
    out->merge = in->merge_factor;
    out->modes = in->modes;
    out->spacing = in->spacing;
    out->origin = in->origin;
    out->period = double(in->site_count) * in->spacing;
    int offset = 0, level = 0;
    for (long long tile = in->base_tile_sites; tile <= in->site_count;
         tile *= in->merge_factor, ++level) {
        if (level >= MAX_LEVELS) {
            snprintf(err, errlen, "too many hierarchy levels");
            return TCST_ERR_UNSUPPORTED;
        }
        for (int k = 0; k < 2; ++k) {
            out->node_offset[2 * level + k] = offset;
            offset += int(in->site_count / tile);
        }
    }
    out->levels = level;
    out->node_count = offset;
    return TCST_OK;
}

__host__ int make_coords(const tcst_coordinates *in, const AxisCfg &out_ax,
                         const AxisCfg &in_ax, CoordCfg *out, char *err, int errlen) {
    if (!in) {
        snprintf(err, errlen, "coordinate declaration is NULL");
        return TCST_ERR_ARGUMENT;
    }
    memset(out, 0, sizeof(*out));
    out->kind = in->kind;
    out->amax = in->amplitude_max;
    if (in->kind == TCST_RATIONAL) {
        out->rmin = in->radius_min;
        out->rbirth = in->radius_birth;
        out->rmax = in->radius_max;
        if (!(in->radius_min > 0) || !(in->radius_min < in->radius_max) ||
            !(in->radius_min <= in->radius_birth && in->radius_birth <= in->radius_max) ||
            !(in->amplitude_max > 0)) {
            snprintf(err, errlen, "invalid rational radius bounds");
            return TCST_ERR_ARGUMENT;
        }
        if (in->radius_max > out_ax.period / 2 || in->radius_max > in_ax.period / 2) {
            snprintf(err, errlen, "radius bounds must fit each chart half-period");
            return TCST_ERR_ARGUMENT;
        }
        // rational_radius.py:113-121: representable float32 clamp interval.
        float lo = float(in->radius_min);
        if (double(lo) < in->radius_min) lo = nextafterf(lo, INFINITY);
        float hi = float(in->radius_max);
        if (double(hi) > in->radius_max) hi = nextafterf(hi, 0.0f);
        if (lo > hi) {
            snprintf(err, errlen, "radius interval has no representable value in parameter dtype");
            return TCST_ERR_ARGUMENT;
        }
        out->lo32 = lo;
        out->hi32 = hi;
    } else if (in->kind == TCST_POLAR) {
        out->w_c = in->w_c;
        out->kappa = in->kappa;
        out->lower_kappa = in->lower_kappa;
        out->udp = in->upper_decay_power;
        for (int i = 0; i < 4; ++i) {
            out->ob[i] = in->out_bounds[i];
            out->ib[i] = in->in_bounds[i];
        }
        if (!(in->amplitude_max > 0) || !(in->w_c > 0) || !(in->kappa > 1) ||
            !(in->upper_decay_power <= 1) || !(in->lower_kappa > 0)) {
            snprintf(err, errlen, "invalid Polar coordinate declaration");
            return TCST_ERR_ARGUMENT;
        }
        if (in->out_bounds[2] > out_ax.period / 2 || in->in_bounds[2] > in_ax.period / 2) {
            snprintf(err, errlen, "radius bounds must fit each chart half-period");
            return TCST_ERR_ARGUMENT;
        }
    } else {
        snprintf(err, errlen, "unknown coordinate kind %d", in->kind);
        return TCST_ERR_ARGUMENT;
    }
    return TCST_OK;
}

// Rational envelope of one Polar side (_backends/torch/parameterizations/
// polar_amp_width.py:206-243, rational branch), float64.
__device__ inline double polar_radius(double amp, double alpha, const double *b,
                                      const CoordCfg &c) {
    double minimum = b[0], birth = b[1], maximum = b[2], floor_ = b[3];
    double ratio = ddiv(amp, c.w_c);
    double x = dmul(ratio, ratio);
    double lower_delta = dsub(birth, minimum);
    double upper_delta = dsub(maximum, minimum);
    double upper_x = c.udp == 1.0 ? x : pow(x, c.udp);
    double upper = dadd(minimum, ddiv(dmul(upper_delta, c.kappa), dadd(c.kappa, upper_x)));
    double lower = dadd(minimum, ddiv(lower_delta, dadd(1.0, dmul(c.lower_kappa, x))));
    upper = fmax(upper, floor_);
    upper = fmax(upper, lower);
    double sigma = exp(dadd(dmul(dsub(1.0, alpha), log(lower)), dmul(alpha, log(upper))));
    return fmin(fmax(sigma, lower), upper);
}

// Chebyshev-square density coefficients on local period P and their radius
// derivative (_backends/torch/profiles/radius_fourier.py:14-58). The reference
// samples the scaled recurrence p_0 = 2, p_1 = u, p_n = u p_{n-1} - (z/4) p_{n-2}
// (u = cos(theta/2), z = cos^2(pi R/P)) at 2M+1 angles, squares it and takes the
// DFT. p_M^2 is an even polynomial of degree 2M in u, hence a trigonometric
// polynomial of degree M in theta, so that DFT is exact and equals a polynomial
// in y = -z/4:  C_k = sum_s W[k][s] y^s, with W built on the host from the
// recurrence's integer coefficients and the binomial Fourier coefficients of
// ((1 + cos theta)/2)^m. The sample scale and the 1/(2M+1) factor cancel in the
// c_0 = 1/P normalization.
struct ProfileTab {
    int modes;
    double w[(MAX_MODES + 1) * (MAX_MODES + 1)]; // w[k * (M + 1) + s]
};

__host__ inline void make_profile_tab(int M, ProfileTab *t) {
    // p_n as coefficients of y^j u^(n-2j), y = -z/4.
    double p[MAX_MODES + 1][MAX_MODES / 2 + 1] = {};
    p[0][0] = 2.0;
    if (M >= 1) p[1][0] = 1.0;
    for (int n = 2; n <= M; ++n)
        for (int j = 0; j <= n / 2; ++j)
            p[n][j] = p[n - 1][j] + (j > 0 ? p[n - 2][j - 1] : 0.0);
    double q[MAX_MODES + 1] = {}; // p_M^2 as coefficients of y^s u^(2M-2s)
    for (int j = 0; j <= M / 2; ++j)
        for (int l = 0; l <= M / 2; ++l)
            if (j + l <= M) q[j + l] += p[M][j] * p[M][l];
    t->modes = M;
    for (int k = 0; k <= M; ++k)
        for (int s = 0; s <= M; ++s) {
            const int m = M - s;
            double v = 0.0;
            if (k <= m) {
                double binom = 1.0; // C(2m, m + k)
                for (int i = 1; i <= m - k; ++i) binom = binom * double(m + k + i) / double(i);
                v = q[s] * binom * std::ldexp(1.0, -2 * m);
            }
            t->w[k * (M + 1) + s] = v;
        }
}

template <int MT>
__device__ inline void write_axis_block_t(float *blk, const Route &r, double R, const AxisCfg &ax,
                                          const ProfileTab &tab) {
    constexpr int CAP = MT > 0 ? MT : MAX_MODES;
    const int M = MT > 0 ? MT : ax.modes;
    const double P = dmul(double(r.count * r.tile), ax.spacing);
    double sa, ca;
    sincospi(R / P, &sa, &ca);
    const double y = -0.25 * ca * ca;
    const double dy = 0.5 * ca * sa * (PI / P); // dy/dR
    // C_k and dC_k/dR one k at a time (Horner in y), so few doubles stay live.
    auto coef = [&](int k, double &c, double &d) {
        const double *w = tab.w + k * (M + 1);
        double v = w[M], dv = 0.0;
        for (int s2 = M - 1; s2 >= 0; --s2) {
            dv = fma(dv, y, v);
            v = fma(v, y, w[s2]);
        }
        c = v;
        d = dv * dy;
    };
    double C0, dC0;
    coef(0, C0, dC0);
    const long long first = (long long)r.first_tile * r.tile;
    const int F = r.count * r.tile;
    const double inv = 1.0 / (P * C0);
    // sin(pi k x1) for k = 0..M by the Chebyshev recurrence
    // sin((k+1)a) = 2 cos(a) sin(k a) - sin((k-1)a), from one sincospi.
    const double x1 = ax.spacing / P;
    double s1, c1;
    sincospi(x1, &s1, &c1);
    double sprev = 0.0, scur = s1;
    // Reciprocals once: sinc_k = sin(pi k x1) / (pi k x1).
    const double inv_pix = 1.0 / (PI * x1), inv_c0 = 1.0 / C0;
    const float phase0 = float(2.0 * (double(first) * ax.spacing - r.local) / P);
    const float omega = float(2.0 * PI / P);
    if constexpr (MT > 0) {
        // Whole block in registers, then float4 stores (the block is 16-byte aligned).
        float w[24];
        w[0] = __int_as_float(int(first));
        w[1] = __int_as_float(F);
        w[2] = phase0;
        w[3] = omega;
#pragma unroll
        for (int k = 0; k <= MT; ++k) {
            double Ck = C0, dCk = dC0, sinc = 1.0;
            if (k > 0) {
                coef(k, Ck, dCk);
                sinc = scur * inv_pix * (1.0 / double(k));
                const double sn = 2.0 * c1 * scur - sprev;
                sprev = scur;
                scur = sn;
            }
            const double wk = (k == 0 ? 1.0 : 2.0) * ax.spacing * sinc;
            w[4 + k] = float(wk * Ck * inv);
            w[5 + MT + k] = float(wk * (dCk * C0 - Ck * dC0) * inv * inv_c0);
        }
#pragma unroll
        for (int k = 6 + 2 * MT; k < 24; ++k) w[k] = 0.f;
        float4 *b4 = reinterpret_cast<float4 *>(blk);
#pragma unroll
        for (int q = 0; q < 6; ++q) b4[q] = make_float4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    } else {
        int *iblk = reinterpret_cast<int *>(blk);
        iblk[0] = int(first);
        iblk[1] = F;
        blk[2] = phase0;
        blk[3] = omega;
#pragma unroll 1
        for (int k = 0; k <= M; ++k) {
            double Ck = C0, dCk = dC0, sinc = 1.0;
            if (k > 0) {
                coef(k, Ck, dCk);
                sinc = scur * inv_pix * (1.0 / double(k));
                const double sn = 2.0 * c1 * scur - sprev;
                sprev = scur;
                scur = sn;
            }
            const double wk = (k == 0 ? 1.0 : 2.0) * ax.spacing * sinc;
            blk[4 + k] = float(wk * Ck * inv);
            blk[5 + M + k] = float(wk * (dCk * C0 - Ck * dC0) * inv * inv_c0);
        }
    }
    (void)CAP;
}

__device__ inline void write_axis_block(float *blk, const Route &r, double R, const AxisCfg &ax,
                                        const ProfileTab &tab) {
    if (ax.modes == 8)
        write_axis_block_t<8>(blk, r, R, ax, tab);
    else
        write_axis_block_t<0>(blk, r, R, ax, tab);
}

// Site values (m, dm/dmu, dm/dR on the first REACH footprint sites of each
// axis) of the atoms of the site classes, from their records: eight threads per
// atom, four per axis, each owning SITE_RUN consecutive sites. cos / sin of
// pi t_j for consecutive sites by rotation from the thread's first site
// (t_j = phase0 + 2 j / F): two sincospif per thread instead of one per site.
// Runs beside the sort, which does not read the site values.
constexpr int SITE_PARTS = 4, SITE_RUN = REACH / SITE_PARTS;
static_assert(SITE_RUN % 4 == 0, "whole float4 chunks per thread");

__global__ void __launch_bounds__(256) site_values_kernel(Table tv) {
    pdl_wait();
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long a = tid / (2 * SITE_PARTS);
    const int side = int(tid / SITE_PARTS) & 1, part = int(tid % SITE_PARTS);
    if (a >= tv.atoms) return;
    const int4 span = tv.spans[a];
    if (span.y <= 0 || span.w <= 0 || max(span.y, span.w) > REACH) return;
    const int F = side ? span.w : span.y, j0 = part * SITE_RUN;
    if (j0 >= F) return;
    AxisCoef<8> ac;
    ac.load(tv.rec + a * (long long)tv.words + 4 + side * axis_words(8));
    float4 *s4 = reinterpret_cast<float4 *>(const_cast<float *>(tv.sites) + a * SITE_FLOATS +
                                            side * 3 * REACH);
    float sj, cj, sd, cd;
    sincospif(ac.phase0 + 2.0f * float(j0) / float(F), &sj, &cj);
    sincospif(2.0f / float(F), &sd, &cd);
#pragma unroll
    for (int q = j0 / 4; q < (j0 + SITE_RUN) / 4; ++q) {
        if (4 * q < F) {
            SiteVals v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                v[u] = ac.values_cs(cj, sj);
                const float cn = fmaf(cj, cd, -sj * sd);
                sj = fmaf(sj, cd, cj * sd);
                cj = cn;
            }
            s4[q] = make_float4(v[0].m, v[1].m, v[2].m, v[3].m);
            s4[REACH / 4 + q] = make_float4(v[0].dmu, v[1].dmu, v[2].dmu, v[3].dmu);
            s4[REACH / 2 + q] = make_float4(v[0].dR, v[1].dR, v[2].dR, v[3].dR);
        }
    }
}

struct Decoded {
    double amp, r_out, r_in, ch0, ch1;
    int flags;
    unsigned bad;
};

// Physical amplitude, radii and chain-rule factors of one atom row. Every lane
// of the warp calls it outside divergent code: lanes 2i and 2i + 1 hold the same
// row and split the rational path's two logarithms and two of its divisions
// (`odd` is the lane's parity), exchanging the results by shuffles.
__device__ inline Decoded decode_atom(float4 row, const CoordCfg &cc, const AxisCfg &out_ax,
                                      const AxisCfg &in_ax, bool odd) {
    Decoded d = {0, 0, 0, 0, 0, 0, 0u};
    if (!(isfinite(row.x) && isfinite(row.y) && isfinite(row.z) && isfinite(row.w)))
        d.bad |= TCST_STATUS_NONFINITE;
    const int lane = threadIdx.x & 31;
    if (cc.kind == TCST_RATIONAL) {
        // _backends/torch/parameterizations/rational_radius.py:6-38.
        const bool fin = !d.bad;
        const double av = row.x, q = row.y;
        double denom = 1.0, lower = 1.0, raw = 0.0;
        if (fin) {
            if (q < 0 || q > 1 || fabs(av) > cc.amax) d.bad |= TCST_STATUS_BOUNDS;
            const double ratio = ddiv(av, 0.3);
            denom = dadd(1.0, dmul(3.0, dmul(ratio, ratio)));
            lower = dadd(cc.rmin, ddiv(dsub(cc.rbirth, cc.rmin), denom));
        }
        // log(lower) on the even lane, log(r_max) on the odd one.
        const double lx = log(odd ? cc.rmax : lower);
        const double log_lower = __shfl_sync(0xffffffffu, lx, lane & ~1);
        const double log_high = __shfl_sync(0xffffffffu, lx, lane | 1);
        if (fin) {
            raw = exp(dadd(dmul(dsub(1.0, q), log_lower), dmul(q, log_high)));
            const double value = q == 0 ? lower : (q == 1 ? cc.rmax : raw);
            float enc = __double2float_rn(value);
            enc = fminf(fmaxf(enc, cc.lo32), cc.hi32);
            d.r_out = d.r_in = double(enc);
            d.amp = av;
        }
        // raw (1 - q) / lower on the even lane, 6 a / 0.09 on the odd one.
        const double quot = odd ? (6.0 * av) / 0.09 : (raw * (1.0 - q)) / lower;
        const double q_even = __shfl_sync(0xffffffffu, quot, lane & ~1);
        const double q_odd = __shfl_sync(0xffffffffu, quot, lane | 1);
        if (fin) {
            const double dlower = -(cc.rbirth - cc.rmin) * q_odd / (denom * denom);
            d.ch0 = q_even * dlower;
            d.ch1 = raw * (log_high - log_lower);
        }
    } else if (!d.bad) {
        // _backends/torch/parameterizations/polar_amp_width.py:127-139.
        const double s = row.x, t = row.y;
        const double rs = dadd(dmul(s, s), dmul(t, t));
        const double tiny = 1.1754943508222875e-38; // float32 tiny: the parameter dtype's
        const double rad = sqrt(fmax(rs, tiny));
        d.amp = ddiv(dmul(cc.amax, s), rad);
        const double alpha = fmin(fmax(ddiv(dsub(rs, 1.0), 3.0), 0.0), 1.0);
        d.r_out = polar_radius(d.amp, alpha, cc.ob, cc);
        d.r_in = polar_radius(d.amp, alpha, cc.ib, cc);
        if (rs > tiny) {
            const double r3 = rad * rad * rad;
            d.ch0 = cc.amax * (1.0 / rad - s * s / r3);
            d.ch1 = -cc.amax * s * t / r3;
        } else {
            d.ch0 = cc.amax / rad;
        }
        d.flags |= 1;
    }
    if (!d.bad && !(d.r_out > 0 && d.r_out <= out_ax.period / 2 && d.r_in > 0 &&
                    d.r_in <= in_ax.period / 2))
        d.bad |= TCST_STATUS_RADIUS;
    return d;
}

// Two threads per atom (adjacent lanes): both decode the row; thread 0 routes
// and profiles the output axis and writes the record header, the output span
// and the owner key; thread 1 does the input axis.
__global__ void __launch_bounds__(256, 4) decode_route_kernel(
    const float *__restrict__ p, AxisCfg out_ax, AxisCfg in_ax, CoordCfg cc,
    const __grid_constant__ ProfileTab tab_out, const __grid_constant__ ProfileTab tab_in,
    Table tv, long long *__restrict__ keys, int *__restrict__ routing,
    unsigned *__restrict__ status) {
    pdl_wait();
    if (blockIdx.x == 0) {
        // The sort's ticket, the active owner-pair count and the node flags.
        if (threadIdx.x == 0) tv.sync[0] = tv.sync[1] = 0u;
        for (int i = threadIdx.x; i < tv.geom.nodes; i += blockDim.x) tv.node_on[i] = 0;
    }
    const long long atoms = tv.atoms;
    const int words = tv.words;
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long a = tid >> 1;
    const int side = int(tid & 1); // 0 = output axis, 1 = input axis
    const bool live = a < atoms;
    const float4 row = live ? reinterpret_cast<const float4 *>(p)[a] : make_float4(0, 0, 0, 0);
    const Decoded d = decode_atom(row, cc, out_ax, in_ax, side != 0);
    const AxisCfg &ax = side ? in_ax : out_ax;
    float *rec = const_cast<float *>(tv.rec) + a * (long long)words;
    float *blk = rec + 4 + (side ? axis_words(out_ax.modes) : 0);
    int4 *spans = const_cast<int4 *>(tv.spans);
    int node = 0, wrapped = 0, foot = 0, lvl = -1, kk = 0;
    if (live && d.bad) {
        if (side == 0) {
            atomicOr(status, d.bad);
            rec[0] = rec[1] = rec[2] = 0.0f;
            reinterpret_cast<int *>(rec)[3] = d.flags | 2;
            spans[a] = make_int4(0, 0, 0, 0);
            tv.bin_of[a] = tv.geom.nbins - 1;
            if (keys) keys[a] = -1;
        }
        reinterpret_cast<int *>(blk)[0] = 0;
        reinterpret_cast<int *>(blk)[1] = 0;
        if (routing)
            for (int i = 0; i < 3; ++i) routing[a * 6 + 3 * side + i] = -1;
    } else if (live) {
        const double R = side ? d.r_in : d.r_out;
        const Route r = route_axis(R, double(side ? row.w : row.z), ax);
        write_axis_block(blk, r, R, ax, side ? tab_in : tab_out);
        {
            const long long first = (long long)r.first_tile * r.tile;
            const long long wr = first % ax.sites;
            wrapped = int(wr < 0 ? wr + ax.sites : wr);
            foot = r.count * r.tile;
        }
        lvl = r.level;
        kk = r.count;
        const int tc = ax.sites / r.tile;
        int m = r.first_tile % tc;
        m += m < 0 ? tc : 0;
        node = ax.node_offset[2 * r.level + r.count - 2] + m;
        if (side == 0) {
            rec[0] = float(d.amp);
            rec[1] = float(d.ch0);
            rec[2] = float(d.ch1);
            reinterpret_cast<int *>(rec)[3] = d.flags;
        }
        if (routing) {
            int *rt = routing + a * 6 + 3 * side;
            rt[0] = r.level;
            rt[1] = r.count;
            rt[2] = r.first_tile;
        }
    }
    // Owner key no * input_node_count + ni (reference pipeline.cu:75-80); the
    // output thread also publishes the span pair and the atom's bin.
    const int other = __shfl_xor_sync(0xffffffffu, node, 1);
    const int other_wrapped = __shfl_xor_sync(0xffffffffu, wrapped, 1);
    const int other_foot = __shfl_xor_sync(0xffffffffu, foot, 1);
    const int other_lvl = __shfl_xor_sync(0xffffffffu, lvl, 1);
    const int other_k = __shfl_xor_sync(0xffffffffu, kk, 1);
    if (live && !d.bad && side == 0) {
        if (keys) keys[a] = (long long)node * in_ax.node_count + other;
        const int4 span = make_int4(wrapped, foot, other_wrapped, other_foot);
        spans[a] = span;
        tv.bin_of[a] = atom_bin(span, tv.geom, lvl, kk, other_lvl, other_k);
    }
}

// Stable counting sort of the atoms by bin, in three launches:
//   count:   sort block b counts the bins of its contiguous atom chunk into
//            counts[b][bin];
//   column:  each bin's column becomes exclusive prefixes over the blocks
//            (counts[b][bin] = atoms of that bin in blocks < b), its total goes
//            to counts[blocks][bin], and the last CTA scans the totals into
//            the bin starts (offsets);
//   scatter: every block walks its chunk in id order and places each atom
//            after the earlier atoms of its bin (warp match + warp-ordered
//            claims), so every bin lists its atoms in id order.
constexpr int SORT_THREADS = 512;

// Per-block bin counters are 16-bit (a block holds at most 65,535 atoms), two
// to a shared-memory word, so the shared histogram covers MAX_BINS bins.
__device__ __forceinline__ unsigned half_add(unsigned *words, int bin, unsigned n) {
    const int shift = (bin & 1) * 16;
    return (atomicAdd(words + (bin >> 1), n << shift) >> shift) & 0xFFFFu;
}

__global__ void __launch_bounds__(SORT_THREADS) bin_count_kernel(Table tv) {
    pdl_wait();
    extern __shared__ unsigned hist[];
    const BinGeom &g = tv.geom;
    const int words = (g.nbins + 1) >> 1;
    for (int i = threadIdx.x; i < words; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const long long a0 = blockIdx.x * g.chunk, a1 = min(tv.atoms, a0 + g.chunk);
    for (long long a = a0 + threadIdx.x; a < a1; a += blockDim.x) half_add(hist, tv.bin_of[a], 1);
    __syncthreads();
    int *row = tv.counts + (long long)blockIdx.x * g.nbins;
    for (int i = threadIdx.x; i < g.nbins; i += blockDim.x)
        row[i] = int((hist[i >> 1] >> ((i & 1) * 16)) & 0xFFFFu);
}

// Column prefix: counts[b][bin] becomes the number of atoms of `bin` in sort
// blocks before b (counts[sort_blocks][bin] = the bin's total). A CTA takes 32
// bins (lanes) and splits the sort blocks into COL_SEGS segments (warps): each
// warp sums its segment, the segment offsets come from shared memory, then the
// warp writes its running prefixes. The last CTA to finish (ticket in
// tv.sync, which the decode reset) scans the totals into the bin starts
// tv.offsets.
constexpr int COL_SEGS = 16;
constexpr int COL_RUN = 16; // segment lengths up to this stay in registers

__global__ void __launch_bounds__(COL_SEGS * 32) bin_column_kernel(Table tv) {
    pdl_wait();
    __shared__ int seg_sum[COL_SEGS][32];
    __shared__ int wsum[COL_SEGS];
    __shared__ bool last;
    const BinGeom &g = tv.geom;
    const int t = threadIdx.x, lane = t & 31, seg = t >> 5;
    const int bin = blockIdx.x * 32 + lane;
    const int per = (g.sort_blocks + COL_SEGS - 1) / COL_SEGS;
    const int b_lo = min(seg * per, g.sort_blocks), b_hi = min(b_lo + per, g.sort_blocks);
    const bool live = bin < g.nbins;
    int *col = tv.counts + bin;
    const long long stride = g.nbins;
    int v[COL_RUN];
    int sum = 0;
    if (live && b_hi - b_lo <= COL_RUN) {
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) v[u] = b_lo + u < b_hi ? col[(b_lo + u) * stride] : 0;
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) sum += v[u];
    } else if (live) {
        for (int b = b_lo; b < b_hi; ++b) sum += col[b * stride];
    }
    seg_sum[seg][lane] = sum;
    __syncthreads();
    int run = 0;
    for (int k = 0; k < seg; ++k) run += seg_sum[k][lane];
    if (live) {
        if (b_hi - b_lo <= COL_RUN) {
#pragma unroll
            for (int u = 0; u < COL_RUN; ++u)
                if (b_lo + u < b_hi) {
                    col[(b_lo + u) * stride] = run;
                    run += v[u];
                }
        } else {
            for (int b = b_lo; b < b_hi; ++b) {
                const int c = col[b * stride];
                col[b * stride] = run;
                run += c;
            }
        }
        if (seg == COL_SEGS - 1) {
            col[g.sort_blocks * stride] = run;
            // Owner pairs: an output node of an expansion level-bank is "on"
            // when one of its pairs holds PAIR_MIN atoms; sync[1] counts the
            // active pairs (both were zeroed by the decode).
            const int l = run >= PAIR_MIN ? pair_lb(g, bin) : -1;
            if (l >= 0 && g.pl_exp[l]) {
                atomicOr(tv.node_on + g.pl_node[l] + (bin - g.pl_base[l]) / g.pl_ni[l], 1);
                atomicAdd(tv.sync + 1, 1u);
            }
        }
    }
    // Last CTA: bin starts = exclusive scan of the totals. The barrier orders
    // this CTA's column writes before thread 0's device-scope fence and ticket
    // (the fence is cumulative), and the last CTA fences after its ticket.
    __syncthreads();
    if (t == 0) {
        __threadfence();
        last = atomicAdd(tv.sync, 1u) == gridDim.x - 1;
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    // Totals of other CTAs are read from L2 (__ldcg), past any stale L1 line,
    // COL_RUN at a time so their latencies overlap.
    const int *total = tv.counts + (long long)g.sort_blocks * g.nbins;
    const int n = g.nbins, nt = blockDim.x;
    const int chunk = (n + nt - 1) / nt, i0 = t * chunk;
    int local = 0;
    for (int k0 = 0; k0 < chunk; k0 += COL_RUN) {
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) {
            const int i = i0 + k0 + u;
            v[u] = k0 + u < chunk && i < n ? __ldcg(total + i) : 0;
        }
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) local += v[u];
    }
    int inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) wsum[seg] = inc;
    __syncthreads();
    int base = inc - local;
    for (int w = 0; w < seg; ++w) base += wsum[w];
    for (int k0 = 0; k0 < chunk; k0 += COL_RUN) {
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) {
            const int i = i0 + k0 + u;
            v[u] = k0 + u < chunk && i < n ? __ldcg(total + i) : 0;
        }
#pragma unroll
        for (int u = 0; u < COL_RUN; ++u) {
            const int i = i0 + k0 + u;
            if (k0 + u < chunk && i < n) {
                tv.offsets[i] = base;
                base += v[u];
            }
        }
    }
    if (t == 0) tv.offsets[n] = int(tv.atoms);
}

// Scatter: every sort block places its atoms at bin start + its column prefix
// + the claims made so far in the block; warps claim one after another, so
// ids stay in increasing order inside every bin.
__global__ void __launch_bounds__(SORT_THREADS) bin_scatter_kernel(Table tv) {
    pdl_wait();
    extern __shared__ unsigned cursor[]; // 16-bit claims made so far, per bin
    const BinGeom &g = tv.geom;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int *mine = tv.counts + (long long)blockIdx.x * g.nbins;
    for (int i = t; i < (g.nbins + 1) >> 1; i += SORT_THREADS) cursor[i] = 0;
    __syncthreads();
    const long long a0 = blockIdx.x * g.chunk, a1 = min(tv.atoms, a0 + g.chunk);
    for (long long base = a0; base < a1; base += SORT_THREADS) {
        const long long a = base + t;
        const bool live = a < a1;
        const int bin = live ? tv.bin_of[a] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, bin);
        const int leader = __ffs(peers) - 1;
        const int rank = __popc(peers & ((1u << lane) - 1u));
        // Loaded before the ordered claims.
        const int bin_base = live ? tv.offsets[bin] + mine[bin] : 0;
        int start = 0;
        for (int w = 0; w < SORT_THREADS / 32; ++w) {
            if (warp == w && live && lane == leader)
                start = bin_base + int(half_add(cursor, bin, unsigned(__popc(peers))));
            __syncthreads();
        }
        start = __shfl_sync(0xffffffffu, start, leader);
        if (live) {
            // The span and amplitude travel with the id, so that readers in
            // sorted order load them beside the id instead of through it.
            const int k = start + rank;
            tv.ids[k] = int(a);
            tv.sspan[k] = tv.spans[a];
            tv.samp[k] = tv.rec[a * tv.words];
        }
    }
}

// Per-atom squared norm of one axis profile with images folded modulo N.
__device__ double axis_energy(const float *blk, int modes, int n) {
    int first = reinterpret_cast<const int *>(blk)[0];
    int F = reinterpret_cast<const int *>(blk)[1];
    double acc = 0;
    if (F <= n) {
        for (int j = 0; j < F; ++j) {
            double m = site_mass(blk, modes, j, F);
            acc += m * m;
        }
        return acc;
    }
    // Longer periods: add the repeated images first, then square
    // (radius_cell_mass.py:162-205).
    for (int site = 0; site < n; ++site) {
        double v = 0;
        int j0 = wrap_site((long long)site - first, n);
        for (int j = j0; j < F; j += n) v += site_mass(blk, modes, j, F);
        acc += v * v;
    }
    return acc;
}

__global__ void energy_kernel(const float *__restrict__ table, int words, long long atoms,
                              AxisCfg out_ax, AxisCfg in_ax, double *__restrict__ energy) {
    pdl_wait();
    long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (a >= atoms) return;
    const float *rec = table + a * (long long)words;
    double amp = rec[0];
    double eo = axis_energy(rec + 4, out_ax.modes, out_ax.sites);
    double ei = axis_energy(rec + 4 + axis_words(out_ax.modes), in_ax.modes, in_ax.sites);
    energy[a] = amp * amp * eo * ei;
}

} // namespace tcst

using namespace tcst;

extern "C" int64_t tcst_atom_table_bytes(int64_t atoms, const tcst_axis *out_axis,
                                         const tcst_axis *in_axis) {
    if (atoms < 0 || !out_axis || !in_axis) return -1;
    // Records, spans, site values, bins, the sort workspace and the owner-pair
    // region (common.cuh).
    return table_layout(atoms, record_words(out_axis->modes, in_axis->modes),
                        axis_geo(*out_axis), axis_geo(*in_axis))
        .total;
}

extern "C" int tcst_decode_route(const float *p_dev, int64_t atoms, const tcst_axis *out_axis,
                                 const tcst_axis *in_axis, const tcst_coordinates *coords,
                                 void *atom_table_dev, int64_t *owner_keys_dev,
                                 int32_t *routing_dev, uint32_t *status_dev, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    CoordCfg cc;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err))) ||
        (rc = make_coords(coords, oa, ia, &cc, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (atoms < 0 || (atoms && (!p_dev || !atom_table_dev || !status_dev))) {
        tcst_set_error("tcst_decode_route: invalid atom count or NULL pointer");
        return TCST_ERR_ARGUMENT;
    }
    if (!atom_table_dev || !status_dev) {
        tcst_set_error("tcst_decode_route: NULL atom table or status word");
        return TCST_ERR_ARGUMENT;
    }
    if (reinterpret_cast<uintptr_t>(p_dev) % 16 || reinterpret_cast<uintptr_t>(atom_table_dev) % 16) {
        tcst_set_error("tcst_decode_route: p and the atom table must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms > 0x7fffffffLL) {
        tcst_set_error("tcst_decode_route: at most 2^31 - 1 atoms");
        return TCST_ERR_UNSUPPORTED;
    }
    const int words = record_words(oa.modes, ia.modes);
    const Table tv = table_view(atom_table_dev, atoms, words, axis_geo(oa), axis_geo(ia));
    const BinGeom &g = tv.geom;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t hist_bytes = size_t((g.nbins + 1) >> 1) * 4;
    static bool configured = false;
    if (!configured) {
        TCST_CUDA(cudaFuncSetAttribute(bin_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       MAX_BINS * 2));
        TCST_CUDA(cudaFuncSetAttribute(bin_scatter_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_BINS * 2));
        configured = true;
    }
    if (atoms == 0) {
        TCST_CUDA(cudaMemsetAsync(tv.offsets, 0, size_t(g.nbins + 1) * 4, st));
        TCST_CUDA(cudaMemsetAsync(tv.sync, 0, 16, st));
        return TCST_OK;
    }
    {
        const int threads = 256;
        const long long blocks = (2 * atoms + threads - 1) / threads;
        ProfileTab to, ti;
        make_profile_tab(oa.modes, &to);
        make_profile_tab(ia.modes, &ti);
        TCST_CUDA(launch_pdl(decode_route_kernel, dim3(unsigned(blocks)), dim3(threads), 0, st, 
            p_dev, oa, ia, cc, to, ti, tv, (long long *)owner_keys_dev, routing_dev, status_dev));
        TCST_CUDA(cudaGetLastError());
    }
    // The site values of the site classes on a side stream, beside the sort
    // (binned geometries only: they have eight modes on both axes).
    SideStreams side(st, g.nclass > 0 ? 1 : 0);
    rc = side.status();
    if (!rc && g.nclass > 0) {
        const long long threads = 2LL * SITE_PARTS * atoms;
        const cudaError_t e = launch_pdl(site_values_kernel, dim3(unsigned((threads + 255) / 256)),
                                         dim3(256), 0, side[0], tv);
        if (e != cudaSuccess) rc = tcst_cuda_check(e, "site_values_kernel");
    }
    cudaError_t e = cudaSuccess;
    if (!rc) e = launch_pdl(bin_count_kernel, dim3(unsigned(g.sort_blocks)), dim3(SORT_THREADS), hist_bytes, st, tv);
    if (!rc && e == cudaSuccess)
        e = launch_pdl(bin_column_kernel, dim3(unsigned((g.nbins + 31) / 32)), dim3(COL_SEGS * 32), 0, st, tv);
    if (!rc && e == cudaSuccess)
        e = launch_pdl(bin_scatter_kernel, dim3(unsigned(g.sort_blocks)), dim3(SORT_THREADS), hist_bytes, st, tv);
    if (!rc && e != cudaSuccess) rc = tcst_cuda_check(e, "bin sort");
    const int rj = side.join();
    return rc ? rc : rj;
}

extern "C" int tcst_atom_energies(const void *atom_table_dev, int64_t atoms,
                                  const tcst_axis *out_axis, const tcst_axis *in_axis,
                                  double *energy_dev, void *stream) {
    char err[256];
    AxisCfg oa, ia;
    int rc;
    if ((rc = make_axis(out_axis, &oa, err, sizeof(err))) ||
        (rc = make_axis(in_axis, &ia, err, sizeof(err)))) {
        tcst_set_error("%s", err);
        return rc;
    }
    if (atoms < 0 || (atoms && (!atom_table_dev || !energy_dev))) {
        tcst_set_error("tcst_atom_energies: invalid atom count or NULL pointer");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    int words = record_words(oa.modes, ia.modes);
    TCST_CUDA(launch_pdl(energy_kernel, dim3(unsigned((atoms + 127) / 128)), dim3(128), 0, (cudaStream_t)stream, 
        (const float *)atom_table_dev, words, atoms, oa, ia, energy_dev));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
