// Host and device copies of one compressor's tables (R, codebook, Phi).
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"
#include "kernels.h"

namespace lc {

void lloyd_max(uint32_t bits, uint64_t n_iter, std::vector<double>& boundaries, std::vector<double>& centroids);
void haar_rotation(uint64_t dim, uint64_t seed, std::vector<float>& R);
void gaussian_projection(uint64_t dim, uint64_t m, uint64_t seed, std::vector<float>& P);

struct Codec {
  uint64_t dim = 0;
  uint32_t bits = 0;
  uint64_t m = 0;
  std::vector<float> R;        // [dim*dim] row-major
  std::vector<double> bounds;  // [2^bits + 1]
  std::vector<double> cents;   // [2^bits]
  std::vector<float> P;        // [m*dim] row-major

  static Codec generate(uint32_t bits, uint64_t m, uint64_t seed, uint64_t n_iter, uint64_t dim);
  static Codec from_tables(uint64_t dim, uint32_t bits, uint64_t m, const float* R, const double* b,
                           const double* cents, const float* P);
  static Codec from_files(const char* cb_path, const char* rot_path, const char* qjl_path);
  void save(const char* cb_path, const char* rot_path, const char* qjl_path) const;
  uint64_t words() const { return (dim + (64 / bits) - 1) / (64 / bits); }
  uint64_t qwords() const { return (m + 63) / 64; }
};

// Device tables in the layouts the kernels read.
struct CodecOnDevice {
  int dim = 0, bits = 0, m = 0;
  // Scale for the f16 centroid tables of the tensor-core decode: alpha*c_k
  // rounds to f16 with the smallest worst-case relative error over the
  // codebook (1 when not searched). Scores and outputs divide it back out.
  float alpha = 1.0f;
  // Largest |alpha c_k - f16(alpha c_k)| over the codebook (alpha c_k taken in
  // f32, as the kernels form it): the scale of the f16 table's rounding,
  // which the decode's score-precision test weighs against the query norm.
  float lo_max = 0.0f;
  float* R = nullptr;
  float* RTd = nullptr;
  float* PTd = nullptr;
  float* thr_d = nullptr;
  float* cent_d = nullptr;
  void upload(const Codec& c);
  void free();
  CodecDev view() const;
  ~CodecOnDevice() { free(); }
};

}  // namespace lc

// The opaque ABI handle of one compressor's tables.
struct lc_codec {
  lc::Codec c;
};
