// Seeded data of the hot path: modular-arithmetic equation tables with their
// split and abstract-symbol permutation (src/gpt/grokking.rs:95-306) and the
// Zipf token streams of the Mesh GPT benchmark shapes (inverse CDF on the
// reference's SplitMix64 Random, src/mesh.rs:256-288).

#include <cmath>

#include "host.h"

namespace mb {

namespace {

uint32_t modular_inverse(uint64_t value, uint64_t p) {
  // Fermat's little theorem by square-and-multiply (src/gpt/grokking.rs:95-107)
  uint64_t result = 1, base = value, e = p - 2;
  while (e) {
    if (e & 1) result = result * base % p;
    base = base * base % p;
    e >>= 1;
  }
  return (uint32_t)result;
}

uint32_t apply(uint32_t op, uint64_t a, uint64_t b, uint64_t p) {
  // src/gpt/grokking.rs:55-67
  switch (op) {
    case 0: return (uint32_t)((a + b) % p);
    case 1: return (uint32_t)(a * b % p);
    case 2: return (uint32_t)((a + p - b) % p);
    case 3: return (uint32_t)(a * modular_inverse(b, p) % p);
    case 4: return b % 2 == 1 ? (uint32_t)(a * modular_inverse(b, p) % p) : (uint32_t)((a + p - b) % p);
    case 5: return (uint32_t)((a * a + b * b) % p);
    case 6: return (uint32_t)((a * a + a * b + b * b) % p);
    case 7: return (uint32_t)((a * a + a * b + b * b + a) % p);
    case 8: return (uint32_t)((a * a * a + a * b) % p);
    case 9: return (uint32_t)((a * a * a + a * b * b + b) % p);
  }
  throw Error(MB_ERR_INVALID, "unknown operation");
}

}  // namespace

void equation_dataset(uint32_t modulus, uint32_t operation, double fraction, uint64_t seed,
                      std::vector<uint32_t>& residues, std::vector<Equation>& train, std::vector<Equation>& valid) {
  bool prime = modulus >= 2 && modulus <= 254;
  for (uint32_t d = 2; prime && d < modulus; ++d) prime = modulus % d != 0;
  require(prime, "modulus must be a prime in 2..254 (two vocabulary slots are reserved)");
  require(std::isfinite(fraction) && fraction > 0.0 && fraction < 1.0,
          "train fraction must be finite and strictly between 0 and 1");
  require(operation <= 9, "unknown operation");
  residues.resize(modulus);
  for (uint32_t i = 0; i < modulus; ++i) residues[i] = i;
  Random symbols(seed ^ 0x73796d626f6c7301ull);
  shuffle(residues, symbols);
  std::vector<Equation> all;
  const uint32_t first_b = operation == 3 ? 1 : 0;
  for (uint32_t a = 0; a < modulus; ++a)
    for (uint32_t b = first_b; b < modulus; ++b) all.push_back(Equation{a, b, apply(operation, a, b, modulus)});
  const size_t split = (size_t)std::floor((double)all.size() * fraction);
  require(split >= 2 && split < all.size(), "split needs at least two training equations and one validation equation");
  Random splits(seed ^ 0x73706c6974730002ull);
  shuffle(all, splits);
  train.assign(all.begin(), all.begin() + split);
  valid.assign(all.begin() + split, all.end());
}

void zipf_batch(uint64_t base_seed, uint32_t rank, uint64_t step, size_t sequences, size_t context,
                uint32_t vocab, double exponent, uint32_t* inputs, uint32_t* targets) {
  require(vocab >= 1 && context >= 1 && std::isfinite(exponent), "invalid Zipf stream shape");
  // cdf[k] = (sum_{j<=k} j^-s) / (sum_{j<=V} j^-s), sequential sums.
  std::vector<double> cdf(vocab);
  double total = 0.0;
  for (uint32_t k = 1; k <= vocab; ++k) {
    total += std::pow((double)k, -exponent);
    cdf[k - 1] = total;
  }
  for (auto& c : cdf) c /= total;
  Random random(base_seed + 1000003ull * rank + step);
  std::vector<uint32_t> stream(context + 1);
  for (size_t s = 0; s < sequences; ++s) {
    for (size_t i = 0; i <= context; ++i) {
      const double u = (double)random.unit();
      uint32_t lo = 0, hi = vocab;  // first index with cdf > u
      while (lo < hi) {
        uint32_t mid = (lo + hi) / 2;
        if (cdf[mid] > u) hi = mid; else lo = mid + 1;
      }
      stream[i] = lo < vocab ? lo : vocab - 1;
    }
    for (size_t i = 0; i < context; ++i) {
      inputs[s * context + i] = stream[i];
      targets[s * context + i] = stream[i + 1];
    }
  }
}

}  // namespace mb
