// TEST INFRASTRUCTURE ONLY. This file is the CPU oracle that the parity tests,
// `__graft_entry__.smoke()` and `bench.py`'s cpu_baseline leg use as the
// checker. Nothing on the product path links, loads or calls it.
//
// It restates, in C++, the reference's CPU TurboQuant path
// (rabbitson87/lumen-rs):
//   crates/lumen-core/src/lloyd_max.rs   -> orc_lloyd_max, orc_codebook_mse
//   crates/lumen-core/src/rotation.rs    -> orc_rotation_*
//   crates/lumen-core/src/bitpack.rs     -> orc_packed_words, orc_pack_codes, orc_unpack_codes
//   crates/lumen-core/src/qjl.rs         -> orc_qjl_*
//   crates/lumen-core/src/compressor.rs  -> orc_compress_one, orc_estimate_*
//   crates/turboquant-cache/src/simple.rs -> orc_sc_* (SimpleCache)
// following the reference's f32/f64 operation order exactly: no FMA contraction
// (build with -ffp-contract=off), left-to-right sequential sums, f64 codebook
// compares. Rust's f32 `Iterator::sum` folds from -0.0; the oracle does the
// same (the sign of an all-zero sum never reaches a code, a QJL bit or a norm).
//
// Parity pins: the reference's own unit-test thresholds (codebook MSE and
// symmetry, bitpack word counts, QJL packed_len and last-word masking,
// compressor cosine bounds, SimpleCache value cosine and compression ratio)
// are re-run against this file by tests/test_oracle_codec.py. The reference
// draws R and Phi from rand 0.10 StdRng / rand_distr 0.6 StandardNormal, whose
// streams cannot be reproduced here; the oracle therefore takes R, Phi and the
// codebook as explicit tables (the reference's TQRM/TQJL/TQCB files, see
// crates/lumen-core/src/compressor.rs:43-58 `from_files`) and offers its own
// documented generator (SplitMix64 + Box-Muller) for test inputs. The Haar
// construction itself (MGS + sign fix, rotation.rs:47-87) is restated.

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <algorithm>

extern "C" {

// ---------------------------------------------------------------------------
// Seeded generator for tables and test inputs (not the reference's StdRng).
// SplitMix64 as in crates/lumen-mlx/src/native_cache/golden_tests.rs:25-36.
// ---------------------------------------------------------------------------
uint64_t orc_splitmix_next(uint64_t* state) {
    *state += 0x9e3779b97f4a7c15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

// Standard normal f64 by Box-Muller over two 53-bit uniforms; u1 in (0, 1].
static double gauss_f64(uint64_t* st) {
    double u1 = (double)((orc_splitmix_next(st) >> 11) + 1) * (1.0 / 9007199254740992.0);
    double u2 = (double)(orc_splitmix_next(st) >> 11) * (1.0 / 9007199254740992.0);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

void orc_gauss_f64(uint64_t seed, double* out, int64_t n) {
    uint64_t st = seed;
    for (int64_t i = 0; i < n; ++i) out[i] = gauss_f64(&st);
}

void orc_gauss_f32(uint64_t seed, float* out, int64_t n) {
    uint64_t st = seed;
    for (int64_t i = 0; i < n; ++i) out[i] = (float)gauss_f64(&st);
}

// ---------------------------------------------------------------------------
// Lloyd-Max codebook for N(0,1): crates/lumen-core/src/lloyd_max.rs:33-122.
// ---------------------------------------------------------------------------
static const double ORC_PI = 3.14159265358979323846;
static const double ORC_FRAC_1_SQRT_2 = 0.70710678118654752440;

static double signum_f64(double x) {  // Rust f64::signum (NaN -> NaN)
    if (std::isnan(x)) return x;
    return std::signbit(x) ? -1.0 : 1.0;
}

// lloyd_max.rs:35-37
static double phi(double x) { return std::exp(-0.5 * x * x) / std::sqrt(2.0 * ORC_PI); }

// lloyd_max.rs:46-54 (Abramowitz & Stegun 7.1.26, not libm erf)
static double erf_as(double x) {
    double sign = signum_f64(x);
    x = std::fabs(x);
    double t = 1.0 / (1.0 + 0.3275911 * x);
    double poly = t * (0.254829592 +
                       t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 + t * 1.061405429))));
    return sign * (1.0 - poly * std::exp(-x * x));
}

// lloyd_max.rs:41-43
static double capital_phi(double x) { return 0.5 * (1.0 + erf_as(x * ORC_FRAC_1_SQRT_2)); }

// lloyd_max.rs:61-67
static double conditional_expectation(double a, double b) {
    double prob = capital_phi(b) - capital_phi(a);
    if (prob < 1e-15) return 0.5 * (a + b);
    return (phi(a) - phi(b)) / prob;
}

// lloyd_max.rs:74-122. boundaries: n+1 values, centroids: n values.
int orc_lloyd_max(int bits, int n_iter, double* boundaries, double* centroids) {
    if (bits == 0 || bits > 8) return -1;
    int n = 1 << bits;
    for (int i = 0; i < n; ++i) centroids[i] = -3.0 + 6.0 * ((double)i + 0.5) / (double)n;
    for (int i = 0; i <= n; ++i) boundaries[i] = 0.0;
    for (int it = 0; it < n_iter; ++it) {
        boundaries[0] = -INFINITY;
        boundaries[n] = INFINITY;
        for (int i = 1; i < n; ++i) boundaries[i] = 0.5 * (centroids[i - 1] + centroids[i]);
        for (int i = 0; i < n; ++i) centroids[i] = conditional_expectation(boundaries[i], boundaries[i + 1]);
    }
    int half = n / 2;
    for (int i = 0; i < half; ++i) {
        double avg = 0.5 * (std::fabs(centroids[i]) + std::fabs(centroids[n - 1 - i]));
        centroids[i] = -avg;
        centroids[n - 1 - i] = avg;
    }
    boundaries[0] = -INFINITY;
    boundaries[n] = INFINITY;
    for (int i = 1; i < n; ++i) boundaries[i] = 0.5 * (centroids[i - 1] + centroids[i]);
    return 0;
}

// lloyd_max.rs:165-185
double orc_codebook_mse(int bits, const double* b, const double* c) {
    int n = 1 << bits;
    double total = 0.0;
    for (int i = 0; i < n; ++i) {
        double a = b[i], bb = b[i + 1];
        double prob = capital_phi(bb) - capital_phi(a);
        if (prob < 1e-15) continue;
        double ci = c[i];
        double ex = (phi(a) - phi(bb)) / prob;
        double a_phi = std::isfinite(a) ? a * phi(a) : 0.0;
        double b_phi = std::isfinite(bb) ? bb * phi(bb) : 0.0;
        double ex2 = 1.0 + (a_phi - b_phi) / prob;
        total += prob * (ex2 - 2.0 * ci * ex + ci * ci);
    }
    return total;
}

// lloyd_max.rs:132-143: linear scan, f64 compare.
int orc_quantize(const double* boundaries, int bits, double x) {
    int n = 1 << bits;
    for (int i = 1; i < n; ++i)
        if (x < boundaries[i]) return i - 1;
    return n - 1;
}

// ---------------------------------------------------------------------------
// Rotation: crates/lumen-core/src/rotation.rs:35-128
// ---------------------------------------------------------------------------

// rotation.rs:47-87 (MGS + Mezzadri sign fix + row-major f32), fed with a
// caller-supplied column-major Gaussian matrix `cols` (dim*dim f64, column j
// at cols[j*dim ..]); the reference draws it from StdRng(seed).
void orc_rotation_from_gaussian(int dim, const double* gauss_cols, float* matrix) {
    std::vector<std::vector<double>> cols(dim, std::vector<double>(dim));
    for (int j = 0; j < dim; ++j)
        for (int i = 0; i < dim; ++i) cols[j][i] = gauss_cols[(size_t)j * dim + i];
    std::vector<double> r_diag(dim, 0.0);
    for (int j = 0; j < dim; ++j) {
        for (int k = 0; k < j; ++k) {
            double dot = -0.0;  // f64 Iterator::sum
            for (int i = 0; i < dim; ++i) dot += cols[k][i] * cols[j][i];
            for (int i = 0; i < dim; ++i) cols[j][i] -= dot * cols[k][i];
        }
        double ss = -0.0;
        for (int i = 0; i < dim; ++i) ss += cols[j][i] * cols[j][i];
        double norm = std::sqrt(ss);
        r_diag[j] = norm;
        double inv_norm = 1.0 / norm;
        for (int i = 0; i < dim; ++i) cols[j][i] *= inv_norm;
    }
    for (int j = 0; j < dim; ++j) {
        double sign = signum_f64(r_diag[j]);
        for (int i = 0; i < dim; ++i) cols[j][i] *= sign;
    }
    for (int i = 0; i < dim; ++i)
        for (int j = 0; j < dim; ++j) matrix[(size_t)i * dim + j] = (float)cols[j][i];
}

// Haar rotation from the oracle's own seeded stream (column-major fill, as
// rotation.rs:39-45 fills `cols`).
void orc_rotation_generate(int dim, uint64_t seed, float* matrix) {
    std::vector<double> g((size_t)dim * dim);
    orc_gauss_f64(seed, g.data(), (int64_t)g.size());
    orc_rotation_from_gaussian(dim, g.data(), matrix);
}

// rotation.rs:91-99: y[i] = sum_j R[i*d+j]*x[j], ascending j.
void orc_rotation_apply(const float* R, int dim, const float* x, float* y) {
    for (int i = 0; i < dim; ++i) {
        const float* row = R + (size_t)i * dim;
        float acc = -0.0f;
        for (int j = 0; j < dim; ++j) acc = acc + row[j] * x[j];
        y[i] = acc;
    }
}

// rotation.rs:102-113: j-outer accumulation into x (starts at +0.0).
void orc_rotation_apply_inverse(const float* R, int dim, const float* y, float* x) {
    for (int i = 0; i < dim; ++i) x[i] = 0.0f;
    for (int j = 0; j < dim; ++j) {
        float yj = y[j];
        const float* row = R + (size_t)j * dim;
        for (int i = 0; i < dim; ++i) x[i] = x[i] + row[i] * yj;
    }
}

// ---------------------------------------------------------------------------
// Bit packing: crates/lumen-core/src/bitpack.rs:11-52
// ---------------------------------------------------------------------------
int orc_packed_words(int n, int bits) {
    int cpw = 64 / bits;
    return (n + cpw - 1) / cpw;
}

void orc_pack_codes(const uint8_t* codes, int n, int bits, uint64_t* packed) {
    int cpw = 64 / bits;
    int nw = orc_packed_words(n, bits);
    for (int w = 0; w < nw; ++w) packed[w] = 0;
    for (int i = 0; i < n; ++i) {
        int word = i / cpw;
        int off = (i % cpw) * bits;
        packed[word] |= (uint64_t)codes[i] << off;
    }
}

void orc_unpack_codes(const uint64_t* packed, int n, int bits, uint8_t* codes) {
    int cpw = 64 / bits;
    uint64_t mask = (1ULL << bits) - 1;
    for (int i = 0; i < n; ++i) {
        int word = i / cpw;
        int off = (i % cpw) * bits;
        codes[i] = (uint8_t)((packed[word] >> off) & mask);
    }
}

// ---------------------------------------------------------------------------
// QJL: crates/lumen-core/src/qjl.rs:40-119
// ---------------------------------------------------------------------------
int orc_qjl_packed_len(int m) { return (m + 63) / 64; }

// qjl.rs:40-51 shape (m x dim, N(0,1) * 1/sqrt(m) in f32) from the oracle's
// own seeded stream.
void orc_qjl_generate(int dim, int m, uint64_t seed, float* proj) {
    float scale = 1.0f / std::sqrt((float)m);
    uint64_t st = seed;
    for (int64_t i = 0; i < (int64_t)m * dim; ++i) proj[i] = (float)gauss_f64(&st) * scale;
}

// qjl.rs:57-74
void orc_qjl_project_and_pack(const float* proj, int m, int dim, const float* res, uint64_t* packed) {
    int nw = orc_qjl_packed_len(m);
    for (int w = 0; w < nw; ++w) packed[w] = 0;
    for (int r = 0; r < m; ++r) {
        const float* row = proj + (size_t)r * dim;
        float dot = -0.0f;
        for (int j = 0; j < dim; ++j) dot = dot + row[j] * res[j];
        if (dot >= 0.0f) packed[r / 64] |= 1ULL << (r % 64);
    }
}

// qjl.rs:76-84
void orc_qjl_project_query(const float* proj, int m, int dim, const float* q, float* out) {
    for (int r = 0; r < m; ++r) {
        const float* row = proj + (size_t)r * dim;
        float dot = -0.0f;
        for (int j = 0; j < dim; ++j) dot = dot + row[j] * q[j];
        out[r] = dot;
    }
}

// qjl.rs:86-119
float orc_qjl_correction_from_projection(int m, const float* pq, const uint64_t* packed, float rnorm) {
    if (rnorm < 1e-10f) return 0.0f;
    float sum = 0.0f;
    for (int r = 0; r < m; ++r) {
        float s = ((packed[r / 64] >> (r % 64)) & 1ULL) ? 1.0f : -1.0f;
        sum = sum + s * pq[r];
    }
    float scale = rnorm * std::sqrt((float)1.5707963267948966) / std::sqrt((float)m);
    return scale * sum;
}

// ---------------------------------------------------------------------------
// Compressor: crates/lumen-core/src/compressor.rs:20-184
// ---------------------------------------------------------------------------
struct orc_compressor {
    int dim, bits, m;
    std::vector<float> R;         // dim*dim row-major
    std::vector<double> bounds;   // n+1
    std::vector<double> cents;    // n
    std::vector<float> proj;      // m*dim
};

orc_compressor* orc_compressor_new(int dim, int bits, int m, const float* R, const double* bounds,
                                   const double* cents, const float* proj) {
    auto* c = new orc_compressor;
    c->dim = dim; c->bits = bits; c->m = m;
    int n = 1 << bits;
    c->R.assign(R, R + (size_t)dim * dim);
    c->bounds.assign(bounds, bounds + n + 1);
    c->cents.assign(cents, cents + n);
    c->proj.assign(proj, proj + (size_t)m * dim);
    return c;
}

void orc_compressor_free(orc_compressor* c) { delete c; }

int orc_compressor_words(const orc_compressor* c) { return orc_packed_words(c->dim, c->bits); }

// compressor.rs:61-107. Outputs: stage1 (packed_words), stage2 (packed_len(m)),
// residual norm, scale; `codes` (dim bytes) may be null.
void orc_compress_one(const orc_compressor* c, const float* vec, uint64_t* stage1, uint64_t* stage2,
                      float* rnorm, float* scale_out, uint8_t* codes_out) {
    const int dim = c->dim;
    std::vector<float> rotated(dim), deq(dim), recon(dim), residual(dim);
    std::vector<uint8_t> codes(dim);
    orc_rotation_apply(c->R.data(), dim, vec, rotated.data());
    float norm_sq = -0.0f;
    for (int i = 0; i < dim; ++i) norm_sq = norm_sq + rotated[i] * rotated[i];
    float scale = std::sqrt(norm_sq / (float)dim);
    if (scale < 1e-10f) {
        for (int i = 0; i < dim; ++i) codes[i] = 0;
    } else {
        float inv = 1.0f / scale;
        for (int i = 0; i < dim; ++i) codes[i] = (uint8_t)orc_quantize(c->bounds.data(), c->bits, (double)(rotated[i] * inv));
    }
    for (int i = 0; i < dim; ++i) deq[i] = (float)c->cents[codes[i]] * scale;
    orc_rotation_apply_inverse(c->R.data(), dim, deq.data(), recon.data());
    float res_sq = 0.0f;
    for (int i = 0; i < dim; ++i) {
        residual[i] = vec[i] - recon[i];
        res_sq = res_sq + residual[i] * residual[i];
    }
    *rnorm = std::sqrt(res_sq);
    orc_qjl_project_and_pack(c->proj.data(), c->m, dim, residual.data(), stage2);
    orc_pack_codes(codes.data(), dim, c->bits, stage1);
    *scale_out = scale;
    if (codes_out) std::memcpy(codes_out, codes.data(), dim);
}

// compressor.rs:110-116 over n vectors [n, dim].
void orc_compress(const orc_compressor* c, const float* vecs, int64_t n, uint64_t* stage1, uint64_t* stage2,
                  float* rnorm, float* scale) {
    int w1 = orc_packed_words(c->dim, c->bits), w2 = orc_qjl_packed_len(c->m);
    for (int64_t i = 0; i < n; ++i)
        orc_compress_one(c, vecs + i * c->dim, stage1 + i * w1, stage2 + i * w2, rnorm + i, scale + i, nullptr);
}

// compressor.rs:165-184: stage-1 scores.
void orc_estimate_stage1(const orc_compressor* c, const float* query, int64_t n, const uint64_t* stage1,
                         const float* scale, float* out) {
    const int dim = c->dim, w1 = orc_packed_words(dim, c->bits);
    std::vector<float> rq(dim);
    std::vector<uint8_t> codes(dim);
    orc_rotation_apply(c->R.data(), dim, query, rq.data());
    for (int64_t t = 0; t < n; ++t) {
        orc_unpack_codes(stage1 + t * w1, dim, c->bits, codes.data());
        float acc = -0.0f;
        for (int j = 0; j < dim; ++j) acc = acc + rq[j] * (float)c->cents[codes[j]];
        out[t] = acc * scale[t];
    }
}

// compressor.rs:122-159: stage-1 + QJL correction.
void orc_estimate_two_stage(const orc_compressor* c, const float* query, int64_t n, const uint64_t* stage1,
                            const float* scale, const uint64_t* stage2, const float* rnorm, float* out) {
    const int dim = c->dim, w2 = orc_qjl_packed_len(c->m);
    std::vector<float> pq(c->m);
    orc_estimate_stage1(c, query, n, stage1, scale, out);
    orc_qjl_project_query(c->proj.data(), c->m, dim, query, pq.data());
    for (int64_t t = 0; t < n; ++t)
        out[t] = out[t] + orc_qjl_correction_from_projection(c->m, pq.data(), stage2 + t * w2, rnorm[t]);
}

// ---------------------------------------------------------------------------
// SimpleCache: crates/turboquant-cache/src/simple.rs:13-185
// (separate K and V compressors so K and V may use different bit widths).
// ---------------------------------------------------------------------------
struct orc_cv_list {
    std::vector<uint64_t> s1, s2;
    std::vector<float> rnorm, scale;
    int64_t n = 0;
};

struct orc_simple_cache {
    const orc_compressor* kc;
    const orc_compressor* vc;
    int n_layers, n_heads, dim;
    std::vector<orc_cv_list> keys, values;  // [layer*n_heads + head]
};

orc_simple_cache* orc_sc_new(const orc_compressor* kc, const orc_compressor* vc, int n_layers, int n_heads, int dim) {
    auto* s = new orc_simple_cache;
    s->kc = kc; s->vc = vc; s->n_layers = n_layers; s->n_heads = n_heads; s->dim = dim;
    s->keys.resize((size_t)n_layers * n_heads);
    s->values.resize((size_t)n_layers * n_heads);
    return s;
}

void orc_sc_free(orc_simple_cache* s) { delete s; }

static void cv_append(const orc_compressor* c, orc_cv_list& l, const float* x, int64_t n) {
    int w1 = orc_packed_words(c->dim, c->bits), w2 = orc_qjl_packed_len(c->m);
    size_t o1 = l.s1.size(), o2 = l.s2.size(), on = l.rnorm.size();
    l.s1.resize(o1 + n * w1);
    l.s2.resize(o2 + n * w2);
    l.rnorm.resize(on + n);
    l.scale.resize(on + n);
    orc_compress(c, x, n, l.s1.data() + o1, l.s2.data() + o2, l.rnorm.data() + on, l.scale.data() + on);
    l.n += n;
}

// simple.rs:123-135
void orc_sc_store(orc_simple_cache* s, int layer, int head, const float* keys, const float* values, int64_t n) {
    size_t i = (size_t)layer * s->n_heads + head;
    cv_append(s->kc, s->keys[i], keys, n);
    cv_append(s->vc, s->values[i], values, n);
}

int64_t orc_sc_seq_len(const orc_simple_cache* s, int layer, int head) {
    return s->keys[(size_t)layer * s->n_heads + head].n;
}

// simple.rs:137-140
void orc_sc_attend_keys(const orc_simple_cache* s, int layer, int head, const float* query, float* out) {
    const orc_cv_list& l = s->keys[(size_t)layer * s->n_heads + head];
    orc_estimate_stage1(s->kc, query, l.n, l.s1.data(), l.scale.data(), out);
}

// The two-stage scores of a (layer, head)'s keys: estimate_inner_products
// (compressor.rs:122-159) over the stored stage-1 words, scales, QJL words
// and residual norms. SimpleCache itself scores with stage 1 only.
void orc_sc_attend_keys_qjl(const orc_simple_cache* s, int layer, int head, const float* query, float* out) {
    const orc_cv_list& l = s->keys[(size_t)layer * s->n_heads + head];
    orc_estimate_two_stage(s->kc, query, l.n, l.s1.data(), l.scale.data(), l.s2.data(), l.rnorm.data(), out);
}

// simple.rs:76-99 + 142-155: per-token un-rotation of c*sigma*w.
void orc_sc_attend_values(const orc_simple_cache* s, int layer, int head, const float* weights, float* out) {
    const orc_cv_list& l = s->values[(size_t)layer * s->n_heads + head];
    const orc_compressor* c = s->vc;
    const int dim = s->dim, bits = c->bits, cpw = 64 / bits, w1 = orc_packed_words(dim, bits);
    const uint64_t mask = (1ULL << bits) - 1;
    for (int i = 0; i < dim; ++i) out[i] = 0.0f;
    for (int64_t t = 0; t < l.n; ++t) {
        float w = weights[t];
        if (std::fabs(w) < 1e-10f) continue;
        const uint64_t* words = l.s1.data() + t * w1;
        float sc = l.scale[t] * w;
        for (int j = 0; j < dim; ++j) {
            int code = (int)((words[j / cpw] >> ((j % cpw) * bits)) & mask);
            float yj = (float)c->cents[code] * sc;
            const float* row = c->R.data() + (size_t)j * dim;
            for (int i = 0; i < dim; ++i) out[i] = out[i] + row[i] * yj;
        }
    }
}

void orc_sc_clear(orc_simple_cache* s) {
    for (auto& l : s->keys) l = orc_cv_list();
    for (auto& l : s->values) l = orc_cv_list();
}

// simple.rs:174-185
static void cv_truncate(const orc_compressor* c, orc_cv_list& l, int64_t n_keep) {
    if (l.n <= n_keep) return;
    int w1 = orc_packed_words(c->dim, c->bits), w2 = orc_qjl_packed_len(c->m);
    l.n = n_keep;
    l.s1.resize(n_keep * w1);
    l.s2.resize(n_keep * w2);
    l.rnorm.resize(n_keep);
    l.scale.resize(n_keep);
}

void orc_sc_truncate(orc_simple_cache* s, int layer, int64_t n_keep) {
    for (int h = 0; h < s->n_heads; ++h) {
        cv_truncate(s->kc, s->keys[(size_t)layer * s->n_heads + h], n_keep);
        cv_truncate(s->vc, s->values[(size_t)layer * s->n_heads + h], n_keep);
    }
}

// config.rs:48-55 size_bytes summed as simple.rs:102-119.
int64_t orc_sc_memory_bytes(const orc_simple_cache* s) {
    int64_t total = 0;
    for (int side = 0; side < 2; ++side) {
        const auto& lists = side ? s->values : s->keys;
        const orc_compressor* c = side ? s->vc : s->kc;
        int64_t per = (int64_t)orc_packed_words(c->dim, c->bits) * 8 + (int64_t)orc_qjl_packed_len(c->m) * 8 + 4 + 4 + 8 + 4;
        for (const auto& l : lists) total += l.n * per;
    }
    return total;
}

// Copy one (layer, head)'s stored vectors out: the CompressedVector fields.
void orc_sc_read(const orc_simple_cache* s, int layer, int head, int side, uint64_t* s1, uint64_t* s2,
                 float* rnorm, float* scale) {
    const orc_cv_list& l = side ? s->values[(size_t)layer * s->n_heads + head] : s->keys[(size_t)layer * s->n_heads + head];
    if (s1) std::memcpy(s1, l.s1.data(), l.s1.size() * 8);
    if (s2) std::memcpy(s2, l.s2.data(), l.s2.size() * 8);
    if (rnorm) std::memcpy(rnorm, l.rnorm.data(), l.rnorm.size() * 4);
    if (scale) std::memcpy(scale, l.scale.data(), l.scale.size() * 4);
}

// Append already-compressed vectors to (layer, head) of one side (0 = K,
// 1 = V): the CompressedVector fields laid out as orc_sc_read returns them.
// Lets a timing run attend over vectors compressed elsewhere.
void orc_sc_load(orc_simple_cache* s, int layer, int head, int side, int64_t n, const uint64_t* s1,
                 const uint64_t* s2, const float* rnorm, const float* scale) {
  orc_cv_list& l = side ? s->values[(size_t)layer * s->n_heads + head] : s->keys[(size_t)layer * s->n_heads + head];
  const orc_compressor* c = side ? s->vc : s->kc;
  const int w1 = orc_packed_words(c->dim, c->bits), w2 = orc_qjl_packed_len(c->m);
  l.s1.insert(l.s1.end(), s1, s1 + n * w1);
  if (s2) l.s2.insert(l.s2.end(), s2, s2 + n * w2);
  else l.s2.resize(l.s2.size() + n * w2, 0);
  if (rnorm) l.rnorm.insert(l.rnorm.end(), rnorm, rnorm + n);
  else l.rnorm.resize(l.rnorm.size() + n, 0.0f);
  l.scale.insert(l.scale.end(), scale, scale + n);
  l.n += n;
}

// ---------------------------------------------------------------------------
// Decode attention composed from the trait calls the way a caller does:
// scores = attend_keys(q) * scale, w = softmax(scores) (max-subtracted, f64
// normaliser), out = attend_values(w). One (layer, kv-head, query) per call.
// ---------------------------------------------------------------------------
// qjl != 0: score with the two-stage estimate (orc_sc_attend_keys_qjl).
void orc_sc_attend_ex(const orc_simple_cache* s, int layer, int head, const float* query, float scale, int qjl,
                      float* out) {
    const orc_cv_list& l = s->keys[(size_t)layer * s->n_heads + head];
    std::vector<float> sc(l.n > 0 ? l.n : 1), w(l.n > 0 ? l.n : 1);
    if (qjl) orc_sc_attend_keys_qjl(s, layer, head, query, sc.data());
    else orc_sc_attend_keys(s, layer, head, query, sc.data());
    double mx = -INFINITY;
    for (int64_t t = 0; t < l.n; ++t) mx = std::max(mx, (double)sc[t] * (double)scale);
    double sum = 0.0;
    for (int64_t t = 0; t < l.n; ++t) sum += std::exp((double)sc[t] * (double)scale - mx);
    for (int64_t t = 0; t < l.n; ++t) w[t] = (float)(std::exp((double)sc[t] * (double)scale - mx) / sum);
    if (l.n == 0) { for (int i = 0; i < s->dim; ++i) out[i] = 0.0f; return; }
    orc_sc_attend_values(s, layer, head, w.data(), out);
}

void orc_sc_attend(const orc_simple_cache* s, int layer, int head, const float* query, float scale, float* out) {
    orc_sc_attend_ex(s, layer, head, query, scale, 0, out);
}

// Causal prefill: attention over the first n_keys stored tokens only
// (softmax over those scores; the weights of later tokens are zero, which
// attend_values skips).
void orc_sc_attend_prefix(const orc_simple_cache* s, int layer, int head, const float* query, float scale,
                          int64_t n_keys, float* out) {
    const orc_cv_list& l = s->keys[(size_t)layer * s->n_heads + head];
    if (n_keys > l.n) n_keys = l.n;
    std::vector<float> sc(l.n > 0 ? l.n : 1), w(l.n > 0 ? l.n : 1, 0.0f);
    if (n_keys <= 0) { for (int i = 0; i < s->dim; ++i) out[i] = 0.0f; return; }
    orc_sc_attend_keys(s, layer, head, query, sc.data());
    double mx = -INFINITY;
    for (int64_t t = 0; t < n_keys; ++t) mx = std::max(mx, (double)sc[t] * (double)scale);
    double sum = 0.0;
    for (int64_t t = 0; t < n_keys; ++t) sum += std::exp((double)sc[t] * (double)scale - mx);
    for (int64_t t = 0; t < n_keys; ++t) w[t] = (float)(std::exp((double)sc[t] * (double)scale - mx) / sum);
    orc_sc_attend_values(s, layer, head, w.data(), out);
}

// Attention over a subset of the stored tokens (mask[t] != 0): the dense
// decode of the chosen pages in page-sparse decode (sdpa over the gathered
// keys, native_attention.rs:273-293).
void orc_sc_attend_mask(const orc_simple_cache* s, int layer, int head, const float* query, float scale,
                        const uint8_t* mask, float* out) {
    const orc_cv_list& l = s->keys[(size_t)layer * s->n_heads + head];
    std::vector<float> sc(l.n > 0 ? l.n : 1), w(l.n > 0 ? l.n : 1, 0.0f);
    if (l.n == 0) { for (int i = 0; i < s->dim; ++i) out[i] = 0.0f; return; }
    orc_sc_attend_keys(s, layer, head, query, sc.data());
    double mx = -INFINITY;
    for (int64_t t = 0; t < l.n; ++t)
        if (mask[t]) mx = std::max(mx, (double)sc[t] * (double)scale);
    double sum = 0.0;
    for (int64_t t = 0; t < l.n; ++t)
        if (mask[t]) sum += std::exp((double)sc[t] * (double)scale - mx);
    for (int64_t t = 0; t < l.n; ++t)
        if (mask[t]) w[t] = (float)(std::exp((double)sc[t] * (double)scale - mx) / sum);
    orc_sc_attend_values(s, layer, head, w.data(), out);
}

// ---------------------------------------------------------------------------
// RoPE as lc_append_rope applies it before the compressor: token t at
// position pos0 + t, pair i < rot_dims / 2 turned by
// pos * base^(-2i / rot_dims) (angle in f64, cos and sin rounded to f32),
// pairs (i, i + rot_dims / 2) or, traditional, (2i, 2i + 1); f32 products
// and one f32 sum / difference per output, in that order.
// ---------------------------------------------------------------------------
void orc_rope(float* x, int64_t n, int dim, int rot_dims, int64_t pos0, double base, int traditional) {
    const int half = rot_dims / 2;
    for (int64_t t = 0; t < n; ++t) {
        float* v = x + t * dim;
        const int64_t pos = pos0 + t;
        for (int i = 0; i < half; ++i) {
            const double ang = (double)pos * std::pow(base, -2.0 * i / rot_dims);
            const float c = (float)std::cos(ang), s = (float)std::sin(ang);
            const int i0 = traditional ? 2 * i : i, i1 = traditional ? 2 * i + 1 : i + half;
            const float x0 = v[i0], x1 = v[i1];
            const float a = x0 * c, b = x1 * s, p = x0 * s, q = x1 * c;
            v[i0] = a - b;
            v[i1] = p + q;
        }
    }
}

// ---------------------------------------------------------------------------
// FNV-1a (golden_tests.rs:73-84), for the ring-digest model.
// ---------------------------------------------------------------------------
uint64_t orc_fnv1a(uint64_t h, const uint8_t* p, int64_t n) {
    for (int64_t i = 0; i < n; ++i) h = (h ^ (uint64_t)p[i]) * 0x100000001b3ULL;
    return h;
}

}  // extern "C"
