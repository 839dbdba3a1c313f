// lumina_selftest: the packed GEMV of every kind against an exact host model
// of the same arithmetic, run before the library is trusted (the role of
// tops._self_test, tops.py:152-238).
#include <cmath>
#include <cstring>
#include <random>
#include <vector>

#include "weights.cuh"

using namespace lumina;

namespace {

// Host restatement of the device arithmetic: int16 activation blocks, exact
// integer dot, per-block fp32 scale-up (see gemv.cu).
double host_gemv_row(const std::vector<int>& codes, const std::vector<float>& scales, int cols, int group,
                     int bits, const std::vector<float>& x, int r) {
  const int L = (1 << bits) - 1;
  const int nblk = (cols + 31) / 32, ng = (cols + group - 1) / group;
  double acc = 0.0;
  for (int b = 0; b < nblk; ++b) {
    float amax = 0.f;
    for (int j = 0; j < 32 && b * 32 + j < cols; ++j) amax = std::max(amax, std::fabs(x[b * 32 + j]));
    if (amax == 0.f) continue;
    const float f = 32767.f / amax, sx = amax / 32767.f;
    long d = 0, xs = 0;
    for (int j = 0; j < 32 && b * 32 + j < cols; ++j) {
      const int q = (int)std::nearbyint(x[b * 32 + j] * f);
      d += (long)q * codes[(size_t)r * cols + b * 32 + j];
      xs += q;
    }
    acc += (double)(2 * d - L * xs) * sx * scales[(size_t)r * ng + (b * 32) / group];
  }
  return acc / L;
}

int pack_file(int bits, const std::vector<int>& codes, int rows, int cols, std::vector<uint8_t>& blob,
              int& pack) {
  blob.clear();
  if (bits == 4) {
    pack = LUMINA_PACK_NIBBLE;
    const int st = (cols + 1) / 2;
    blob.assign((size_t)rows * st, 0);
    for (int r = 0; r < rows; ++r)
      for (int k = 0; k < cols; ++k) blob[(size_t)r * st + k / 2] |= codes[(size_t)r * cols + k] << (4 * (k & 1));
  } else if (bits == 2) {
    pack = LUMINA_PACK_2BIT;
    const int st = (cols + 3) / 4;
    blob.assign((size_t)rows * st, 0);
    for (int r = 0; r < rows; ++r)
      for (int k = 0; k < cols; ++k) blob[(size_t)r * st + k / 4] |= codes[(size_t)r * cols + k] << (2 * (k & 3));
  } else if (bits == 1) {
    pack = LUMINA_PACK_NONE;
    const int st = (cols + 7) / 8;
    blob.assign((size_t)rows * st, 0);
    for (int r = 0; r < rows; ++r)
      for (int k = 0; k < cols; ++k) blob[(size_t)r * st + k / 8] |= codes[(size_t)r * cols + k] << (k & 7);
  } else {
    pack = LUMINA_PACK_NONE;
    blob.resize((size_t)rows * cols);
    for (size_t i = 0; i < blob.size(); ++i) blob[i] = (uint8_t)codes[i];
  }
  return 0;
}

}  // namespace

extern "C" int lumina_selftest(int device) {
  int n = 0;
  if (lumina_device_count(&n) || device < 0 || device >= n) {
    set_error("selftest: device %d not available (%d visible)", device, n);
    return LUMINA_E_ARG;
  }
  std::mt19937 rng(11);
  std::uniform_real_distribution<float> U(-1.f, 1.f);
  const int rows = 37, cols = 256 + 96;
  for (int bits = 1; bits <= 4; ++bits) {
    const int group = bits >= 3 ? 64 : 128;
    const int ng = (cols + group - 1) / group;
    std::vector<int> codes((size_t)rows * cols);
    for (auto& c : codes) c = (int)(rng() % (1u << bits));
    std::vector<float> scales((size_t)rows * ng);
    for (auto& s : scales) s = __half2float(__float2half_rn(0.01f + 0.02f * std::fabs(U(rng))));
    std::vector<uint8_t> blob;
    int pack = 0;
    pack_file(bits, codes, rows, cols, blob, pack);
    lumina_weight* w = nullptr;
    int rc = lumina_weight_upload(device, bits, group, pack, blob.data(), blob.size(), scales.data(),
                                  scales.size(), rows, cols, &w);
    if (rc) return rc;
    std::vector<float> x(cols), y(rows);
    for (auto& v : x) v = U(rng);
    rc = lumina_gemv_host(w, x.data(), 1, y.data());
    lumina_weight_free(w);
    if (rc) return rc;
    for (int r = 0; r < rows; ++r) {
      const double ref = host_gemv_row(codes, scales, cols, group, bits, x, r);
      if (std::fabs(y[r] - ref) > 1e-5 * (1.0 + std::fabs(ref))) {
        set_error("selftest: int%d row %d got %.9g want %.9g", bits, r, (double)y[r], ref);
        return LUMINA_E_SELFTEST;
      }
    }
  }
  return LUMINA_OK;
}
