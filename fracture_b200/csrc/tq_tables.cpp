// Host-side TurboQuant tables: Lloyd-Max codebook and Haar rotation matrix.
//
// Restates crates/fracture-core/src/turboquant.rs so a C or C++ caller gets
// the same tables the reference engine uploads (quantized_paged_kv_cache.rs:
// 141-171). All arithmetic is IEEE double in the reference's order (sequential
// sums, no fused multiply-add: this file is compiled with -ffp-contract=off),
// with glibc's exp/log/sqrt/cos/sin/pow as the reference's f64 methods use, so
// the float32 results are bit-identical.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "fracture_b200.h"

namespace {

// turboquant.rs:166-169
double gaussian_pdf(double x, double sigma2) {
    return (1.0 / sqrt(2.0 * M_PI * sigma2)) * exp(-x * x / (2.0 * sigma2));
}

// Composite Simpson's rule (turboquant.rs:172-182); kind 0: x*pdf(x), 1: pdf(x).
double integrate_simpson(int kind, double sigma2, double a, double b, int n) {
    if (n % 2 == 1) n += 1;
    const double h = (b - a) / (double)n;
    auto f = [&](double x) { return kind == 0 ? x * gaussian_pdf(x, sigma2) : gaussian_pdf(x, sigma2); };
    double sum = f(a) + f(b);
    for (int i = 1; i < n; ++i) {
        const double x = a + (double)i * h;
        sum += (i % 2 == 0) ? 2.0 * f(x) : 4.0 * f(x);
    }
    return sum * h / 3.0;
}

// Xoshiro256** seeded by SplitMix64 (turboquant.rs:349-385).
struct Xoshiro256 {
    uint64_t s[4];
    explicit Xoshiro256(uint64_t seed) {
        uint64_t sm = seed;
        for (int i = 0; i < 4; ++i) {
            sm += 0x9e3779b97f4a7c15ULL;
            uint64_t z = sm;
            z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
            z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
            z ^= z >> 31;
            s[i] = z;
        }
    }
    static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
    uint64_t next_u64() {
        const uint64_t result = rotl(s[1] * 5, 7) * 9;
        const uint64_t t = s[1] << 17;
        s[2] ^= s[0];
        s[3] ^= s[1];
        s[1] ^= s[2];
        s[0] ^= s[3];
        s[2] ^= t;
        s[3] = rotl(s[3], 45);
        return result;
    }
    double next_f64() { return (double)(next_u64() >> 11) / (double)(1ULL << 53); }
};

// Box-Muller (turboquant.rs:388-394).
void box_muller(Xoshiro256& rng, float* z0, float* z1) {
    double u1 = rng.next_f64();
    if (u1 < 1e-15) u1 = 1e-15;
    const double u2 = rng.next_f64();
    const double r = sqrt(-2.0 * log(u1));
    const double th = 2.0 * M_PI * u2;
    *z0 = (float)(r * cos(th));
    *z1 = (float)(r * sin(th));
}

}  // namespace

// LloydMaxCodebook::compute (turboquant.rs:186-250).
extern "C" int fb_tq_codebook(int dim, int bits, float* centroids, float* boundaries) {
    if (dim <= 0 || bits < 1 || bits > 8) return 1;
    const int n = 1 << bits;
    const double sigma2 = 1.0 / (double)dim;
    const double sigma = sqrt(sigma2);
    const double lo = -3.5 * sigma, hi = 3.5 * sigma;
    std::vector<double> c(n), b(n > 1 ? n - 1 : 0), nc(n);
    for (int i = 0; i < n; ++i) c[i] = lo + (hi - lo) * ((double)i + 0.5) / (double)n;
    for (int iter = 0; iter < 200; ++iter) {
        for (int i = 0; i + 1 < n; ++i) b[i] = (c[i] + c[i + 1]) / 2.0;
        const double elo = lo * 3.0, ehi = hi * 3.0;
        double max_shift = 0.0;
        for (int i = 0; i < n; ++i) {
            const double a_ = i == 0 ? elo : b[i - 1];
            const double b_ = i == n - 1 ? ehi : b[i];
            const double num = integrate_simpson(0, sigma2, a_, b_, 500);
            const double den = integrate_simpson(1, sigma2, a_, b_, 500);
            const double v = fabs(den) > 1e-15 ? num / den : c[i];
            const double sh = fabs(v - c[i]);
            if (sh > max_shift) max_shift = sh;
            nc[i] = v;
        }
        c.swap(nc);
        if (max_shift < 1e-10) break;
    }
    for (int i = 0; i < n; ++i)
        if (centroids) centroids[i] = (float)c[i];
    for (int i = 0; i + 1 < n; ++i)
        if (boundaries) boundaries[i] = (float)((c[i] + c[i + 1]) / 2.0);
    return 0;
}

// generate_rotation_matrix (turboquant.rs:306-338) with qr_orthogonalize (:399-438).
extern "C" int fb_tq_rotation_matrix(int d, uint64_t seed, float* out) {
    if (d <= 0 || !out) return 1;
    Xoshiro256 rng(seed);
    const size_t n = (size_t)d * d;
    std::vector<float> g;
    g.reserve(n + 1);
    for (size_t p = 0; p < (n + 1) / 2; ++p) {
        float z0, z1;
        box_muller(rng, &z0, &z1);
        g.push_back(z0);
        if (g.size() < n) g.push_back(z1);
    }
    // cols[col][row] in f64 (modified Gram-Schmidt works on columns).
    std::vector<double> cols(n);
    for (int col = 0; col < d; ++col)
        for (int row = 0; row < d; ++row) cols[(size_t)col * d + row] = (double)g[(size_t)row * d + col];
    for (int i = 0; i < d; ++i) {
        double* ci = &cols[(size_t)i * d];
        double ss = 0.0;
        for (int r = 0; r < d; ++r) ss += ci[r] * ci[r];
        const double norm = sqrt(ss);
        if (norm > 1e-12)
            for (int r = 0; r < d; ++r) ci[r] /= norm;
        for (int j = i + 1; j < d; ++j) {
            double* cj = &cols[(size_t)j * d];
            double dot = 0.0;
            for (int r = 0; r < d; ++r) dot += ci[r] * cj[r];
            for (int r = 0; r < d; ++r) cj[r] -= dot * ci[r];
        }
    }
    for (int row = 0; row < d; ++row)
        for (int col = 0; col < d; ++col) out[(size_t)row * d + col] = (float)cols[(size_t)col * d + row];
    // Positive-diagonal sign fix (turboquant.rs:326-335).
    for (int col = 0; col < d; ++col) {
        if (out[(size_t)col * d + col] < 0.0f)
            for (int row = 0; row < d; ++row) out[(size_t)row * d + col] = -out[(size_t)row * d + col];
    }
    return 0;
}
