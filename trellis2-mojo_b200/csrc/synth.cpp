// Seeded synthetic inputs for tests and benchmarks: perturbed-sphere shells
// and the project RNG (xorshift64* seeded through splitmix64, Box-Muller),
// restated from trellis2_mojo/rng.mojo:17-52 so the same seed gives the
// same stream as the reference's generator.
#include <math.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/t2sc.h"

namespace {
struct Rng {
  uint64_t state;
  explicit Rng(uint64_t seed) {
    uint64_t z = seed + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    state = z ^ (z >> 31);
    if (state == 0) state = 0x9E3779B97F4A7C15ULL;
  }
  uint64_t next_u64() {
    uint64_t x = state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    state = x;
    return x * 0x2545F4914F6CDD1DULL;
  }
  double next_f64() { return (double)(next_u64() >> 11) * (1.0 / 9007199254740992.0); }
  double normal() {
    double u1 = next_f64();
    while (u1 == 0.0) u1 = next_f64();
    double u2 = next_f64();
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
  }
};
}  // namespace

extern "C" int t2sc_synth_shell(int g, double radius, double half_width, uint64_t seed, int batch, int32_t *coords,
                                int64_t cap, int64_t *n) {
  if (g <= 0 || g > 4096 || !n || batch < 0) return T2SC_ERR_INVALID;
  double phase = 0.0;
  if (seed != 0) {
    Rng r(seed);
    phase = 6.283185307179586 * r.next_f64();
  }
  const double c = g / 2.0;
  const double rlo = radius * 0.9 - half_width - 1.0, rhi = radius * 1.1 + half_width + 1.0;
  unsigned nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  std::vector<std::vector<int32_t>> parts(g);
  auto work = [&](int t) {
    for (int x = t; x < g; x += nt) {
      std::vector<int32_t> &out = parts[x];
      const double dx = x - c;
      for (int y = 0; y < g; y++) {
        const double dy = y - c;
        for (int z = 0; z < g; z++) {
          const double dz = z - c;
          const double r = sqrt(dx * dx + dy * dy + dz * dz);
          if (r < rlo || r > rhi) continue;
          const double th = r > 0 ? acos(dz / r) : 0.0;
          const double ph = atan2(dy, dx) + phase;
          const double rr = radius * (1.0 + 0.1 * sin(3.0 * th) * cos(2.0 * ph));
          if (fabs(r - rr) <= half_width) {
            out.push_back(y);
            out.push_back(z);
          }
        }
      }
    }
  };
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++) th.emplace_back(work, (int)t);
  for (auto &t : th) t.join();
  int64_t total = 0;
  for (int x = 0; x < g; x++) total += (int64_t)parts[x].size() / 2;
  *n = total;
  if (!coords) return T2SC_OK;
  if (total > cap) return T2SC_ERR_CAPACITY;
  int64_t r = 0;
  for (int x = 0; x < g; x++)
    for (size_t i = 0; i < parts[x].size(); i += 2, r++) {
      coords[4 * r] = batch;
      coords[4 * r + 1] = x;
      coords[4 * r + 2] = parts[x][i];
      coords[4 * r + 3] = parts[x][i + 1];
    }
  return T2SC_OK;
}

extern "C" int t2sc_synth_normal(uint64_t seed, float std_, float *out, int64_t count) {
  if (!out || count < 0) return T2SC_ERR_INVALID;
  Rng r(seed);
  for (int64_t i = 0; i < count; i++) out[i] = (float)r.normal() * std_;
  return T2SC_OK;
}

extern "C" int t2sc_synth_bernoulli(uint64_t seed, double p, float *out, int64_t count) {
  if (!out || count < 0) return T2SC_ERR_INVALID;
  Rng r(seed);
  for (int64_t i = 0; i < count; i++) out[i] = r.next_f64() < p ? 1.0f : 0.0f;
  return T2SC_OK;
}
