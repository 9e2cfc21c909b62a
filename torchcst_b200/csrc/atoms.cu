// Per-atom decode, hierarchy routing and Chebyshev-square Fourier profile.
//
// One thread per atom, float64 throughout. Routing (level, K, first tile, owner
// key) reproduces the reference's float64 operation order with non-contracted
// arithmetic, so it is bit-exact whenever exp/log agree in the last ulp.

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

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
// derivative (_backends/torch/profiles/radius_fourier.py:14-58). The sample
// scale and the 1/(2M+1) factor cancel in the c_0 = 1/P normalization, so the
// unscaled squared recurrence is transformed directly.
__device__ inline void profile_coefficients(double R, double P, int M, double *c, double *dc) {
    int n = 2 * M + 1;
    double sa, ca;
    sincospi(R / P, &sa, &ca);
    double ibs = ca * ca;
    double dibs = -2.0 * ca * sa * (PI / P);
    double C[MAX_MODES + 1], dC[MAX_MODES + 1];
    for (int k = 0; k <= M; ++k) C[k] = dC[k] = 0.0;
    for (int j = 0; j < n; ++j) {
        double cosine = cospi(double(j) / n);
        double prev = 2.0, cur = cosine, dprev = 0.0, dcur = 0.0;
        for (int i = 2; i <= M; ++i) {
            double nxt = cosine * cur - ibs * prev * 0.25;
            double dnxt = cosine * dcur - (dibs * prev + ibs * dprev) * 0.25;
            prev = cur;
            cur = nxt;
            dprev = dcur;
            dcur = dnxt;
        }
        double d = cur * cur, dd = 2.0 * cur * dcur;
        // cos(2 pi j k / n) by the Chebyshev recurrence in k.
        double w1 = cospi(2.0 * double(j) / n);
        double wprev = 1.0, wcur = w1;
        C[0] += d;
        dC[0] += dd;
        for (int k = 1; k <= M; ++k) {
            C[k] += d * wcur;
            dC[k] += dd * wcur;
            double wn = 2.0 * w1 * wcur - wprev;
            wprev = wcur;
            wcur = wn;
        }
    }
    for (int k = 0; k <= M; ++k) {
        c[k] = C[k] / (P * C[0]);
        dc[k] = (dC[k] * C[0] - C[k] * dC[0]) / (P * C[0] * C[0]);
    }
}

__device__ inline void write_axis_block(float *blk, const Route &r, double R, const AxisCfg &ax) {
    int M = ax.modes;
    double P = dmul(double(r.count * r.tile), ax.spacing);
    double c[MAX_MODES + 1], dc[MAX_MODES + 1];
    profile_coefficients(R, P, M, c, dc);
    long long first = (long long)r.first_tile * r.tile;
    int *iblk = reinterpret_cast<int *>(blk);
    iblk[0] = int(first);
    iblk[1] = r.count * r.tile;
    blk[2] = float(2.0 * (double(first) * ax.spacing - r.local) / P);
    blk[3] = float(2.0 * PI / P);
    for (int k = 0; k <= M; ++k) {
        double x = double(k) * ax.spacing / P;
        double sinc = k == 0 ? 1.0 : sinpi(x) / (PI * x);
        double w = (k == 0 ? 1.0 : 2.0) * ax.spacing * sinc;
        blk[4 + k] = float(w * c[k]);
        blk[5 + M + k] = float(w * dc[k]);
    }
}

__global__ void decode_route_kernel(const float *__restrict__ p, long long atoms, AxisCfg out_ax,
                                    AxisCfg in_ax, CoordCfg cc, float *__restrict__ table,
                                    int words, long long *__restrict__ keys,
                                    int *__restrict__ routing, unsigned *__restrict__ status) {
    long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (a >= atoms) return;
    float4 row = reinterpret_cast<const float4 *>(p)[a];
    float *rec = table + a * (long long)words;
    int *irec = reinterpret_cast<int *>(rec);
    unsigned bad = 0;
    if (!(isfinite(row.x) && isfinite(row.y) && isfinite(row.z) && isfinite(row.w)))
        bad |= TCST_STATUS_NONFINITE;
    double amp = 0, r_out = 0, r_in = 0, ch0 = 0, ch1 = 0;
    int flags = 0;
    if (!bad && cc.kind == TCST_RATIONAL) {
        // _backends/torch/parameterizations/rational_radius.py:6-38.
        double av = row.x, q = row.y;
        if (q < 0 || q > 1 || fabs(av) > cc.amax) bad |= TCST_STATUS_BOUNDS;
        double ratio = ddiv(av, 0.3);
        double denom = dadd(1.0, dmul(3.0, dmul(ratio, ratio)));
        double lower = dadd(cc.rmin, ddiv(dsub(cc.rbirth, cc.rmin), denom));
        double log_lower = log(lower), log_high = log(cc.rmax);
        double raw = exp(dadd(dmul(dsub(1.0, q), log_lower), dmul(q, log_high)));
        double value = q == 0 ? lower : (q == 1 ? cc.rmax : raw);
        float enc = __double2float_rn(value);
        enc = fminf(fmaxf(enc, cc.lo32), cc.hi32);
        r_out = r_in = double(enc);
        amp = av;
        double dlower = -(cc.rbirth - cc.rmin) * (6.0 * av / 0.09) / (denom * denom);
        ch0 = raw * (1.0 - q) / lower * dlower;
        ch1 = raw * (log_high - log_lower);
    } else if (!bad) {
        // _backends/torch/parameterizations/polar_amp_width.py:127-139.
        double s = row.x, t = row.y;
        double rs = dadd(dmul(s, s), dmul(t, t));
        double tiny = 1.1754943508222875e-38; // float32 tiny: the parameter dtype's
        double safe = fmax(rs, tiny);
        double rad = sqrt(safe);
        amp = ddiv(dmul(cc.amax, s), rad);
        double alpha = fmin(fmax(ddiv(dsub(rs, 1.0), 3.0), 0.0), 1.0);
        r_out = polar_radius(amp, alpha, cc.ob, cc);
        r_in = polar_radius(amp, alpha, cc.ib, cc);
        if (rs > tiny) {
            double r3 = rad * rad * rad;
            ch0 = cc.amax * (1.0 / rad - s * s / r3);
            ch1 = -cc.amax * s * t / r3;
        } else {
            ch0 = cc.amax / rad;
            ch1 = 0.0;
        }
        flags |= 1;
    }
    if (!bad) {
        if (!(r_out > 0 && r_out <= out_ax.period / 2 && r_in > 0 && r_in <= in_ax.period / 2))
            bad |= TCST_STATUS_RADIUS;
    }
    float *ob = rec + 4;
    float *ib = rec + 4 + axis_words(out_ax.modes);
    if (bad) {
        atomicOr(status, bad);
        rec[0] = 0.0f;
        rec[1] = rec[2] = 0.0f;
        irec[3] = flags | 2;
        reinterpret_cast<int *>(ob)[0] = 0;
        reinterpret_cast<int *>(ob)[1] = 0;
        reinterpret_cast<int *>(ib)[0] = 0;
        reinterpret_cast<int *>(ib)[1] = 0;
        if (keys) keys[a] = -1;
        if (routing)
            for (int i = 0; i < 6; ++i) routing[a * 6 + i] = -1;
        return;
    }
    Route ro = route_axis(r_out, double(row.z), out_ax);
    Route ri = route_axis(r_in, double(row.w), in_ax);
    rec[0] = float(amp);
    rec[1] = float(ch0);
    rec[2] = float(ch1);
    irec[3] = flags;
    write_axis_block(ob, ro, r_out, out_ax);
    write_axis_block(ib, ri, r_in, in_ax);
    if (keys) {
        int tco = out_ax.sites / ro.tile, tci = in_ax.sites / ri.tile;
        int mo = ro.first_tile % tco;
        mo += mo < 0 ? tco : 0;
        int mi = ri.first_tile % tci;
        mi += mi < 0 ? tci : 0;
        long long no = out_ax.node_offset[2 * ro.level + ro.count - 2] + mo;
        long long ni = in_ax.node_offset[2 * ri.level + ri.count - 2] + mi;
        keys[a] = no * in_ax.node_count + ni;
    }
    if (routing) {
        int *rt = routing + a * 6;
        rt[0] = ro.level;
        rt[1] = ro.count;
        rt[2] = ro.first_tile;
        rt[3] = ri.level;
        rt[4] = ri.count;
        rt[5] = ri.first_tile;
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
    return atoms * int64_t(record_words(out_axis->modes, in_axis->modes)) * 4;
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
    if (reinterpret_cast<uintptr_t>(p_dev) % 16 || reinterpret_cast<uintptr_t>(atom_table_dev) % 16) {
        tcst_set_error("tcst_decode_route: p and the atom table must be 16-byte aligned");
        return TCST_ERR_ARGUMENT;
    }
    if (atoms == 0) return TCST_OK;
    int words = record_words(oa.modes, ia.modes);
    int threads = 128;
    long long blocks = (atoms + threads - 1) / threads;
    decode_route_kernel<<<unsigned(blocks), threads, 0, (cudaStream_t)stream>>>(
        p_dev, atoms, oa, ia, cc, (float *)atom_table_dev, words, (long long *)owner_keys_dev,
        routing_dev, status_dev);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
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
    energy_kernel<<<unsigned((atoms + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        (const float *)atom_table_dev, words, atoms, oa, ia, energy_dev);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}
