// Codec tables of one TurboQuant compressor: rotation R, Lloyd-Max codebook,
// QJL projection Phi. Host-side setup (the reference computes these once on
// the CPU too); the kernels only ever see the device copies.
//
//   Lloyd-Max for N(0,1)      crates/lumen-core/src/lloyd_max.rs:33-122
//   Haar rotation (MGS)       crates/lumen-core/src/rotation.rs:35-88
//   QJL projection shape      crates/lumen-core/src/qjl.rs:40-51
//   TQCB / TQRM / TQJL files  lloyd_max.rs:187-213, rotation.rs:130-150,
//                             qjl.rs:248-272, binfile.rs:1-70
//
// The reference seeds R and Phi from rand's StdRng, whose stream is not
// reproducible without its sources; this library's own generator is
// SplitMix64 + Box-Muller (documented in lumen_cuda.h). Loading the
// reference's files gives its exact tables.
#include "codec.h"

#include <cmath>
#include <cstring>
#include <fstream>

namespace lc {

namespace {

// ---- Lloyd-Max (lloyd_max.rs:35-67) ----
constexpr double kPi = 3.14159265358979323846;
constexpr double kFrac1Sqrt2 = 0.70710678118654752440;

double signum(double x) {
  if (std::isnan(x)) return x;
  return std::signbit(x) ? -1.0 : 1.0;
}
double pdf(double x) { return std::exp(-0.5 * x * x) / std::sqrt(2.0 * kPi); }
double erf_as(double x) {  // Abramowitz & Stegun 7.1.26, as the reference uses
  const double sign = signum(x);
  x = std::fabs(x);
  const double t = 1.0 / (1.0 + 0.3275911 * x);
  const double poly =
      t * (0.254829592 + t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 + t * 1.061405429))));
  return sign * (1.0 - poly * std::exp(-x * x));
}
double cdf(double x) { return 0.5 * (1.0 + erf_as(x * kFrac1Sqrt2)); }
double cond_mean(double a, double b) {
  const double prob = cdf(b) - cdf(a);
  if (prob < 1e-15) return 0.5 * (a + b);
  return (pdf(a) - pdf(b)) / prob;
}

uint64_t splitmix(uint64_t& s) {
  s += 0x9e3779b97f4a7c15ULL;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
double gauss(uint64_t& s) {
  const double u1 = (double)((splitmix(s) >> 11) + 1) * (1.0 / 9007199254740992.0);
  const double u2 = (double)(splitmix(s) >> 11) * (1.0 / 9007199254740992.0);
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

void write_u32(std::ofstream& f, uint32_t v) { f.write(reinterpret_cast<const char*>(&v), 4); }
uint32_t read_u32(std::ifstream& f) {
  uint32_t v = 0;
  f.read(reinterpret_cast<char*>(&v), 4);
  if (!f) LC_THROW(LC_ERR_IO, "table file truncated");
  return v;
}
template <class T>
void read_arr(std::ifstream& f, T* dst, size_t n) {
  f.read(reinterpret_cast<char*>(dst), (std::streamsize)(n * sizeof(T)));
  if (!f) LC_THROW(LC_ERR_IO, "table file truncated");
}
void expect_magic(std::ifstream& f, const char* magic, const char* path) {
  char m[4];
  f.read(m, 4);
  if (!f) LC_THROW(LC_ERR_IO, std::string("cannot read ") + path);
  if (std::memcmp(m, magic, 4) != 0) LC_THROW(LC_ERR_MAGIC, std::string("bad magic in ") + path);
}

}  // namespace

void lloyd_max(uint32_t bits, uint64_t n_iter, std::vector<double>& b, std::vector<double>& c) {
  if (bits == 0 || bits > 8) LC_THROW(LC_ERR_BITS, "invalid bit width: must be 1..=8");
  const int n = 1 << bits;
  c.assign(n, 0.0);
  b.assign(n + 1, 0.0);
  for (int i = 0; i < n; ++i) c[i] = -3.0 + 6.0 * ((double)i + 0.5) / (double)n;
  for (uint64_t it = 0; it < n_iter; ++it) {
    b[0] = -INFINITY;
    b[n] = INFINITY;
    for (int i = 1; i < n; ++i) b[i] = 0.5 * (c[i - 1] + c[i]);
    for (int i = 0; i < n; ++i) c[i] = cond_mean(b[i], b[i + 1]);
  }
  for (int i = 0; i < n / 2; ++i) {
    const double avg = 0.5 * (std::fabs(c[i]) + std::fabs(c[n - 1 - i]));
    c[i] = -avg;
    c[n - 1 - i] = avg;
  }
  b[0] = -INFINITY;
  b[n] = INFINITY;
  for (int i = 1; i < n; ++i) b[i] = 0.5 * (c[i - 1] + c[i]);
}

void haar_rotation(uint64_t dim, uint64_t seed, std::vector<float>& R) {
  const size_t d = dim;
  std::vector<double> cols(d * d);  // column j at cols[j*d]
  uint64_t s = seed;
  for (size_t k = 0; k < d * d; ++k) cols[k] = gauss(s);
  std::vector<double> rdiag(d);
  for (size_t j = 0; j < d; ++j) {
    double* cj = &cols[j * d];
    for (size_t k = 0; k < j; ++k) {
      const double* ck = &cols[k * d];
      double dot = -0.0;
      for (size_t i = 0; i < d; ++i) dot += ck[i] * cj[i];
      for (size_t i = 0; i < d; ++i) cj[i] -= dot * ck[i];
    }
    double ss = -0.0;
    for (size_t i = 0; i < d; ++i) ss += cj[i] * cj[i];
    const double norm = std::sqrt(ss);
    rdiag[j] = norm;
    const double inv = 1.0 / norm;
    for (size_t i = 0; i < d; ++i) cj[i] *= inv;
  }
  for (size_t j = 0; j < d; ++j) {
    const double sg = signum(rdiag[j]);
    for (size_t i = 0; i < d; ++i) cols[j * d + i] *= sg;
  }
  R.assign(d * d, 0.f);
  for (size_t i = 0; i < d; ++i)
    for (size_t j = 0; j < d; ++j) R[i * d + j] = (float)cols[j * d + i];
}

void gaussian_projection(uint64_t dim, uint64_t m, uint64_t seed, std::vector<float>& P) {
  const float scale = 1.0f / std::sqrt((float)m);
  P.assign(m * dim, 0.f);
  uint64_t s = seed;
  for (size_t k = 0; k < m * dim; ++k) P[k] = (float)gauss(s) * scale;
}

Codec Codec::generate(uint32_t bits, uint64_t m, uint64_t seed, uint64_t n_iter, uint64_t dim) {
  LC_REQUIRE(dim > 0 && dim <= 512 && dim % 32 == 0, LC_ERR_INVALID, "head_dim must be a multiple of 32 up to 512");
  Codec c;
  c.dim = dim;
  c.bits = bits;
  c.m = m;
  lloyd_max(bits, n_iter, c.bounds, c.cents);
  haar_rotation(dim, seed, c.R);
  gaussian_projection(dim, m, seed + 1, c.P);
  return c;
}

Codec Codec::from_tables(uint64_t dim, uint32_t bits, uint64_t m, const float* R, const double* b, const double* cents,
                         const float* P) {
  LC_REQUIRE(bits >= 1 && bits <= 8, LC_ERR_BITS, "invalid bit width: must be 1..=8");
  LC_REQUIRE(dim > 0 && dim <= 512 && dim % 32 == 0, LC_ERR_INVALID, "head_dim must be a multiple of 32 up to 512");
  LC_REQUIRE(R && b && cents, LC_ERR_INVALID, "null table");
  LC_REQUIRE(m == 0 || P, LC_ERR_INVALID, "null qjl projection with qjl_m > 0");
  Codec c;
  c.dim = dim;
  c.bits = bits;
  c.m = m;
  const size_t n = (size_t)1 << bits;
  c.R.assign(R, R + dim * dim);
  c.bounds.assign(b, b + n + 1);
  c.cents.assign(cents, cents + n);
  if (m) c.P.assign(P, P + m * dim);
  return c;
}

// Formats: binfile.rs write_header + arrays, little-endian.
//   TQCB: "TQCB" bits n_levels | boundaries f64[n+1] | centroids f64[n]
//   TQRM: "TQRM" dim           | f32[dim*dim]
//   TQJL: "TQJL" dim m         | f32[m*dim]
Codec Codec::from_files(const char* cb_path, const char* rot_path, const char* qjl_path) {
  LC_REQUIRE(cb_path && rot_path && qjl_path, LC_ERR_INVALID, "null path");
  Codec c;
  {
    std::ifstream f(cb_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot open ") + cb_path);
    expect_magic(f, "TQCB", cb_path);
    c.bits = read_u32(f);
    const uint32_t n = read_u32(f);
    LC_REQUIRE(c.bits >= 1 && c.bits <= 8 && n == (1u << c.bits), LC_ERR_BITS, "codebook bits/n_levels mismatch");
    c.bounds.resize(n + 1);
    c.cents.resize(n);
    read_arr(f, c.bounds.data(), n + 1);
    read_arr(f, c.cents.data(), n);
  }
  {
    std::ifstream f(rot_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot open ") + rot_path);
    expect_magic(f, "TQRM", rot_path);
    c.dim = read_u32(f);
    LC_REQUIRE(c.dim > 0 && c.dim <= 512 && c.dim % 32 == 0, LC_ERR_INVALID, "rotation dim unsupported");
    c.R.resize(c.dim * c.dim);
    read_arr(f, c.R.data(), c.R.size());
  }
  {
    std::ifstream f(qjl_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot open ") + qjl_path);
    expect_magic(f, "TQJL", qjl_path);
    const uint32_t dim = read_u32(f);
    c.m = read_u32(f);
    LC_REQUIRE(dim == c.dim, LC_ERR_INVALID, "qjl dim differs from rotation dim");
    c.P.resize(c.m * c.dim);
    read_arr(f, c.P.data(), c.P.size());
  }
  return c;
}

void Codec::save(const char* cb_path, const char* rot_path, const char* qjl_path) const {
  if (cb_path) {
    std::ofstream f(cb_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot create ") + cb_path);
    f.write("TQCB", 4);
    write_u32(f, bits);
    write_u32(f, 1u << bits);
    f.write(reinterpret_cast<const char*>(bounds.data()), (std::streamsize)(bounds.size() * 8));
    f.write(reinterpret_cast<const char*>(cents.data()), (std::streamsize)(cents.size() * 8));
    LC_REQUIRE(f.good(), LC_ERR_IO, "write failed");
  }
  if (rot_path) {
    std::ofstream f(rot_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot create ") + rot_path);
    f.write("TQRM", 4);
    write_u32(f, (uint32_t)dim);
    f.write(reinterpret_cast<const char*>(R.data()), (std::streamsize)(R.size() * 4));
    LC_REQUIRE(f.good(), LC_ERR_IO, "write failed");
  }
  if (qjl_path) {
    std::ofstream f(qjl_path, std::ios::binary);
    LC_REQUIRE(f.good(), LC_ERR_IO, std::string("cannot create ") + qjl_path);
    f.write("TQJL", 4);
    write_u32(f, (uint32_t)dim);
    write_u32(f, (uint32_t)m);
    f.write(reinterpret_cast<const char*>(P.data()), (std::streamsize)(P.size() * 4));
    LC_REQUIRE(f.good(), LC_ERR_IO, "write failed");
  }
}

// Smallest f32 >= b: for every f32 x, (double)x < b  <=>  x < t.
static float f32_ceil_of(double b) {
  float t = (float)b;
  if ((double)t < b) t = std::nextafter(t, INFINITY);
  return t;
}

// Nearest f16 value of a positive normal-range float (11 significant bits).
static double round_f16(double x) {
  int e = 0;
  std::frexp(x, &e);  // x = m * 2^e, m in [0.5, 1)
  const double ulp = std::ldexp(1.0, e - 11);
  return std::nearbyint(x / ulp) * ulp;
}

// alpha in [1, 2) minimising max_k |f16(alpha c_k) - alpha c_k| / |alpha c_k|.
static float f16_table_scale(const std::vector<double>& cents) {
  std::vector<double> mags;
  for (double v : cents) {
    const double a = std::fabs((double)(float)v);
    if (a > 0) mags.push_back(a);
  }
  if (mags.empty()) return 1.0f;
  double best = 1e30;
  float best_a = 1.0f;
  const int steps = 1 << 18;
  for (int k = 0; k < steps; ++k) {
    const float a = 1.0f + (float)k / steps;
    double worst = 0;
    for (double mg : mags) {
      const double x = (double)((float)mg * a);
      worst = std::max(worst, std::fabs(round_f16(x) - x) / x);
      if (worst >= best) break;
    }
    if (worst < best) {
      best = worst;
      best_a = a;
    }
  }
  return best_a;
}

void CodecOnDevice::upload(const Codec& c) {
  free();
  dim = (int)c.dim;
  bits = (int)c.bits;
  m = (int)c.m;
  const size_t d = c.dim, n = (size_t)1 << c.bits;
  std::vector<float> RT(d * d), PT(d * (c.m ? c.m : 1), 0.f), thr(n > 1 ? n - 1 : 1, 0.f), cent(n);
  for (size_t i = 0; i < d; ++i)
    for (size_t j = 0; j < d; ++j) RT[j * d + i] = c.R[i * d + j];
  for (size_t r = 0; r < c.m; ++r)
    for (size_t j = 0; j < d; ++j) PT[j * c.m + r] = c.P[r * d + j];
  for (size_t k = 1; k < n; ++k) thr[k - 1] = f32_ceil_of(c.bounds[k]);
  for (size_t k = 0; k < n; ++k) cent[k] = (float)c.cents[k];
  auto up = [](float*& dst, const std::vector<float>& v) {
    LC_CUDA(cudaMalloc(&dst, v.size() * sizeof(float)));
    LC_CUDA(cudaMemcpy(dst, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
  };
  up(R, c.R);
  up(RTd, RT);
  up(PTd, PT);
  up(thr_d, thr);
  up(cent_d, cent);
  alpha = c.bits <= 4 ? f16_table_scale(c.cents) : 1.0f;
  lo_max = 0.0f;
  for (size_t k = 0; k < n; ++k) {
    const float x = cent[k] * alpha;  // the f32 product the kernels round to f16
    const double ax = std::fabs((double)x);
    if (ax == 0) continue;
    lo_max = std::max(lo_max, (float)std::fabs(round_f16(ax) - ax));
  }
}

void CodecOnDevice::free() {
  for (float** p : {&R, &RTd, &PTd, &thr_d, &cent_d}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
}

CodecDev CodecOnDevice::view() const {
  CodecDev v;
  v.dim = dim;
  v.bits = bits;
  v.n_levels = 1 << bits;
  v.m = m;
  v.words = (int)((dim + (64 / bits) - 1) / (64 / bits));
  v.qwords = (m + 63) / 64;
  v.R = R;
  v.RT = RTd;
  v.PT = PTd;
  v.thr = thr_d;
  v.cent = cent_d;
  return v;
}

}  // namespace lc
