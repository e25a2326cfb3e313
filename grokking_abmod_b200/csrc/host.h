// Host-side declarations shared by the executor and the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/meshb200.h"

namespace mb {

// An error carrying one of the MB_ERR_* codes; the C ABI converts it into the
// return status and the thread's last-error message.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void require(bool ok, const std::string& message, int code = MB_ERR_INVALID) {
  if (!ok) throw Error(code, message);
}
// The same for a literal message: nothing is built unless the check fails,
// so per-element validation loops cost a compare and a branch.
inline void require(bool ok, const char* message, int code = MB_ERR_INVALID) {
  if (!ok) throw Error(code, message);
}

inline void need(const void* p, const char* what) { require(p != nullptr, std::string(what) + " must not be null"); }

// The calling thread's last status and message (read by mb_last_error).
void set_last_error(int code, const char* message);

// Runs an entry point body, converting exceptions into a status code.
template <class F>
int guarded(F&& f) {
  try {
    f();
    set_last_error(MB_OK, "");
    return MB_OK;
  } catch (const Error& e) {
    set_last_error(e.code, e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error(MB_ERR_INVALID, "host allocation failed");
  } catch (const std::exception& e) {
    set_last_error(MB_ERR_INVALID, e.what());
  }
  return MB_ERR_INVALID;
}

// ---- SplitMix64 (src/mesh.rs:256-288)
struct Random {
  uint64_t state;
  explicit Random(uint64_t seed) : state(seed) {}
  uint64_t next_u64() {
    state += 0x9e3779b97f4a7c15ull;
    uint64_t b = state;
    b = (b ^ (b >> 30)) * 0xbf58476d1ce4e5b9ull;
    b = (b ^ (b >> 27)) * 0x94d049bb133111ebull;
    return b ^ (b >> 31);
  }
  float unit() { return (float)(uint32_t)(next_u64() >> 40) / 16777216.0f; }
  size_t index(size_t bound) {
    const uint64_t b = bound;
    const uint64_t threshold = (0 - b) % b;
    for (;;) {
      uint64_t bits = next_u64();
      if (bits >= threshold) return (size_t)(bits % b);
    }
  }
};

template <class T>
void shuffle(std::vector<T>& v, Random& r) {
  // src/gpt/grokking.rs:267-271
  for (size_t end = v.size(); end-- > 1;) std::swap(v[end], v[r.index(end + 1)]);
}

// ---- configuration and parameter layout (src/gpt/config.rs)
struct Group {
  size_t offset, size;
  int depth;
};

struct BlockGroups {
  int query, key, value, projection, ffn;
};

struct Layout {
  std::vector<Group> groups;
  std::vector<BlockGroups> blocks;
  int embedding = 0;
  size_t count() const { return groups.empty() ? 0 : groups.back().offset + groups.back().size; }
};

void validate_config(const mb_gpt_config& c);            // reference limits (MB_ERR_INVALID)
void validate_kernel_shapes(const mb_gpt_config& c);     // this build's kernels (MB_ERR_UNSUPPORTED)
Layout make_layout(const mb_gpt_config& c);
std::vector<float> initial_parameters(const mb_gpt_config& c, uint64_t seed);
std::vector<float> token_codes(const mb_gpt_config& c);
int mesh_stride(const mb_gpt_config& c, int layer);
// allow_unsupervised: a data-parallel rank's share may hold no supervised
// target; the device checks the count over all ranks instead.
size_t validate_batch(const mb_gpt_config& c, const uint32_t* inputs, const uint32_t* targets, size_t rows,
                      size_t sequence, bool allow_unsupervised = false);
void validate_optimizer(const mb_adamw& o);

// ---- data
struct Equation {
  uint32_t a, b, answer;
};
void equation_dataset(uint32_t modulus, uint32_t operation, double fraction, uint64_t seed,
                      std::vector<uint32_t>& residues, std::vector<Equation>& train, std::vector<Equation>& valid);
void zipf_batch(uint64_t base_seed, uint32_t rank, uint64_t step, size_t sequences, size_t context,
                uint32_t vocab, double exponent, uint32_t* inputs, uint32_t* targets);

}  // namespace mb
