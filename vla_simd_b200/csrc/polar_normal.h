// The reference's seeded noise: std::normal_distribution<float> over
// std::mt19937_64 (Marsaglia's polar method on generate_canonical uniforms,
// the second value of each pair saved for the next call), with the one
// contraction its -mfma -ffp-contract=fast build makes: r2 = fma(x, x, y*y)
// (read from the compiled reference; x = 2u - 1 is exact either way). Octo's
// and SmolVLA's C ABIs draw their noise this way.
#pragma once
#include <cmath>
#include <cstdint>
#include <random>

namespace vsb {

class PolarNormal {
  public:
    explicit PolarNormal(uint64_t seed) : rng_(seed) {}
    float operator()() {
        if (have_saved_) {
            have_saved_ = false;
            return saved_;
        }
        float x, y, r2;
        do {
            x = 2.0f * std::generate_canonical<float, 24>(rng_) - 1.0f;
            y = 2.0f * std::generate_canonical<float, 24>(rng_) - 1.0f;
            r2 = std::fma(x, x, y * y);
        } while (r2 > 1.0f || r2 == 0.0f);
        const float mult = std::sqrt(-2.0f * std::log(r2) / r2);
        saved_ = x * mult;
        have_saved_ = true;
        return y * mult;
    }

  private:
    std::mt19937_64 rng_;
    float saved_ = 0.0f;
    bool have_saved_ = false;
};

}  // namespace vsb
