// grok-simple configuration: validation, parameter groups, seeded
// initialisation and one-hot decoding (host side of the C ABI).
//
// Restates src/simple/mod.rs: SimpleConfig::validate :561-694 (the rules that
// concern the ten architectures of this build; full-mesh-mlp and non-one-hot
// encodings are out), layers :720-756, mesh_layers :758-765, groups
// :871-889, initial_parameters :938-1036 (default near-identity shared
// chain, uniform fan-in embedding) and encode :1039-1055.  Compiled with
// -ffp-contract=off: the f32 uniform draws and the f64 Box-Muller draws
// round exactly as the reference's.

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "simple.h"

namespace mb {
namespace simple {

int parents(const mb_simple_config& c) { return c.connectivity == kOwn ? 1 : 2; }

int stride(const mb_simple_config& c, int layer) {
  // src/simple/mod.rs:178-186 with src/gpt/config.rs:117-122
  if (c.connectivity == kOwn) return 0;
  if (c.connectivity == kNeighbor) return 1;
  const int log2w = 31 - __builtin_clz(c.width);
  return 1 << (layer % log2w);
}

int mesh_layers(const mb_simple_config& c) {
  // src/simple/mod.rs:754-765
  if (c.architecture == kMeshMlp || c.architecture == kTiedConcatMesh) return (int)c.depth - 1;
  if (residual_mesh(c)) return (int)(c.depth * c.mesh_depth);
  if (c.architecture == kFullMesh) return (int)c.depth + 1;
  if (c.architecture == kSharedNeighbor) return (int)(c.embedding_mesh_depth + c.depth);
  return 0;
}

int stored_mesh_layers(const mb_simple_config& c) {
  return c.tied_mesh ? std::min(mesh_layers(c), 1) : mesh_layers(c);
}

uint32_t operand_features(const mb_simple_config& c) {
  switch (c.encoding) {
    case kBinary: {
      uint32_t bits = 0;
      while ((c.modulus - 1) >> bits) ++bits;
      return std::max(bits, 1u);
    }
    case kScalar: return 1;
    case kDiscreteLog: return 2;
    default: return c.modulus;
  }
}

namespace {
// The smallest primitive root (src/simple/mod.rs:444-456), or 0 without one.
uint32_t primitive_root(uint32_t m) {
  std::vector<char> seen(m);
  for (uint32_t root = 1; root < m; ++root) {
    std::fill(seen.begin(), seen.end(), 0);
    uint64_t v = 1;
    for (uint32_t i = 0; i + 1 < m; ++i) {
      seen[v] = 1;
      v = v * root % m;
    }
    bool all = true;
    for (uint32_t k = 1; k < m && all; ++k) all = seen[k] != 0;
    if (all) return root;
  }
  return 0;
}
}  // namespace

std::vector<float> encoding_table(const mb_simple_config& c) {
  const uint32_t m = c.modulus, f = operand_features(c);
  std::vector<float> t((size_t)m * f, 0.0f);
  if (c.encoding == kOneHot) {
    for (uint32_t v = 0; v < m; ++v) t[(size_t)v * f + v] = 1.0f;
  } else if (c.encoding == kBinary) {
    for (uint32_t v = 0; v < m; ++v)
      for (uint32_t bit = 0; bit < f; ++bit) t[(size_t)v * f + bit] = ((v >> bit) & 1u) ? 1.0f : -1.0f;
  } else if (c.encoding == kScalar) {
    const double middle = (double)(m - 1) / 2.0;
    for (uint32_t v = 0; v < m; ++v) t[v] = (float)(((double)v - middle) / middle);
  } else {
    const uint32_t root = primitive_root(m);
    require(root != 0, "discrete logarithms require a prime modulus");
    std::vector<uint32_t> logs(m, 0);
    uint64_t v = 1;
    for (uint32_t e = 0; e + 1 < m; ++e) {
      logs[v] = e;
      v = v * root % m;
    }
    const double middle = (double)(m - 2) / 2.0;
    for (uint32_t k = 0; k < m; ++k) {
      if (k == 0) {
        t[0] = 1.0f;
      } else if (middle != 0.0) {
        t[(size_t)k * 2 + 1] = (float)(((double)logs[k] - middle) / middle);
      }
    }
  }
  return t;
}

std::vector<std::pair<uint32_t, uint32_t>> dense_layers(const mb_simple_config& c) {
  std::vector<std::pair<uint32_t, uint32_t>> l;
  const uint32_t F = operand_features(c);
  if (c.architecture == kMeshMlp || c.architecture == kResidualMesh) {
    l.push_back({2 * F, c.width});
    l.push_back({c.width, c.modulus});
  } else if (tied_concat(c)) {
    // src/simple/mod.rs:727-729: the shared embedding E, the projection of [E a | E b]
    l.push_back({c.modulus, c.width});
    l.push_back({2 * c.width, c.width});
  } else if (c.architecture == kTiedRotaryResidualMesh) {
    l.push_back({c.modulus, c.width});
  } else if (c.architecture == kRotaryDense) {
    l.push_back({c.modulus, c.width});
    for (uint32_t i = 0; i < c.depth; ++i) l.push_back({c.width, c.width});
  } else if (c.architecture == kMlp) {
    // src/simple/mod.rs:716-721: input layer, depth - 1 hidden layers, readout
    l.push_back({2 * F, c.width});
    for (uint32_t i = 1; i < c.depth; ++i) l.push_back({c.width, c.width});
    l.push_back({c.width, c.modulus});
  } else if (c.architecture == kResidualMlp) {
    // src/simple/mod.rs:735-744: input layer, per block (width -> hidden,
    // hidden -> width), readout
    const uint32_t hidden = c.width * c.expansion;
    l.push_back({2 * F, c.width});
    for (uint32_t i = 0; i < c.depth; ++i) {
      l.push_back({c.width, hidden});
      l.push_back({hidden, c.width});
    }
    l.push_back({c.width, c.modulus});
  } else if (c.architecture == kBilinear) {
    // src/simple/mod.rs:745-749: the a embedding, the b embedding, readout
    l.push_back({F, c.width});
    l.push_back({F, c.width});
    l.push_back({c.width, c.modulus});
  }
  return l;
}

std::vector<TwoParentLayer> two_parent_layers(const mb_simple_config& c) {
  std::vector<TwoParentLayer> l;
  if (c.architecture != kFullMesh) return l;
  const uint32_t F = operand_features(c);
  l.push_back({2 * F, c.width, F});
  for (uint32_t layer = 1; layer < c.depth; ++layer) l.push_back({c.width, c.width, (uint32_t)stride(c, layer - 1)});
  l.push_back({c.width, c.modulus, (uint32_t)stride(c, c.depth - 1)});
  return l;
}

std::vector<size_t> groups(const mb_simple_config& c) {
  std::vector<size_t> g;
  if (c.architecture == kFullMesh) {
    for (const auto& l : two_parent_layers(c)) g.push_back(3 * (size_t)l.outputs);
    return g;
  }
  if (c.architecture == kSharedNeighbor) {
    for (uint32_t i = 0; i < c.embedding_mesh_depth; ++i) g.push_back(2 * (size_t)c.width);
    for (uint32_t i = 0; i < c.depth; ++i) g.push_back(3 * (size_t)c.width);
    return g;
  }
  for (auto& d : dense_layers(c)) g.push_back((size_t)d.first * d.second);
  for (int i = 0; i < stored_mesh_layers(c); ++i) g.push_back((size_t)parents(c) * c.width);
  return g;
}

size_t parameter_count(const mb_simple_config& c) {
  size_t n = 0;
  for (size_t g : groups(c)) n += g;
  return n;
}

void validate(const mb_simple_config& c) {
  require(c.architecture <= kFullMesh,
          "architecture must be 0 (mesh-mlp), 1 (tied-rotary-residual-dense-mlp), 2 (shared-neighbor-mesh-mlp), "
          "3 (mlp), 4 (bilinear), 5 (residual-mlp), 6 (residual-mesh-mlp), 7 (tied-concat-residual-mesh-mlp), "
          "8 (tied-rotary-residual-mesh-mlp), 9 (tied-concat-mesh-mlp) or 10 (full-mesh-mlp)",
          MB_ERR_UNSUPPORTED);
  require(c.activation <= kSquare, "activation must be 0 (relu) or 1 (square)");
  require(c.connectivity <= kButterfly, "connectivity must be 0 (own), 1 (neighbor) or 2 (butterfly)");
  require(c.full_mesh_initialization <= 1, "full-mesh initialization must be 0 (kaiming) or 1 (identity-hidden)");
  require(c.modulus >= 2 && c.modulus <= kMaxClasses, "modulus must be in 2..=1024");
  require(c.width >= 1 && c.width <= kMaxWidth, "width must be in 1..=16384");
  if (c.architecture != kBilinear) require(c.depth >= 1 && c.depth <= kMaxDepth, "depth must be in 1..=64");
  if (c.architecture == kResidualMlp)
    require(c.expansion >= 1 && (uint64_t)c.width * c.expansion <= kMaxWidth,
            "residual hidden width must be in 1..=16384");
  if (residual_mesh(c)) require(c.mesh_depth >= 1 && c.mesh_depth <= kMaxDepth, "mesh depth must be in 1..=64");
  if (c.architecture == kSharedNeighbor)
    require(c.embedding_mesh_depth >= 1 && c.embedding_mesh_depth <= kMaxDepth,
            "shared Neighbor embedding depth must be in 1..=64");
  require(c.mesh_output_activation <= 1, "mesh output activation must be 0 or 1");
  if (c.mesh_output_activation)
    require(residual_mesh(c), "only residual mesh branches activate their final mesh output");
  require(c.tied_mesh <= 1, "tied mesh must be 0 or 1");
  require(c.encoding <= kDiscreteLog, "encoding must be 0 (one-hot), 1 (binary), 2 (scalar) or 3 (discrete-log)");
  if (c.encoding != kOneHot)
    require(c.architecture == kMlp || c.architecture == kMeshMlp || c.architecture == kBilinear ||
                c.architecture == kResidualMlp || c.architecture == kResidualMesh || c.architecture == kFullMesh,
            "this architecture needs one-hot operand encoding");
  if (c.encoding == kDiscreteLog) require(primitive_root(c.modulus) != 0, "discrete logarithms require a prime modulus");
  require(c.decay_factors >= 2, "weight decay imitates at least two factors per channel");
  if (c.decay_factors != 2)
    require(c.architecture == kMlp && c.depth == 1, "only one-layer MLPs decay as more factors per channel");
  if (c.tied_mesh)
    require(c.architecture == kMeshMlp || c.architecture == kTiedConcatMesh, "only mesh MLPs tie mesh layers");
  if (mesh_layers(c) > 0 && parents(c) == 2) require(c.width >= 2, "a second mesh parent needs a width of at least 2");
  if (tied_concat(c))
    require(2 * (uint64_t)c.width <= kMaxWidth, "tied concatenation needs one-hot encoding and width <= 8192");
  if (c.architecture == kRotaryDense || c.architecture == kSharedNeighbor || c.architecture == kTiedRotaryResidualMesh)
    require(c.width >= 2 && c.width % 2 == 0, "rotary roles need one-hot encoding and a positive even width");
  if (c.full_mesh_initialization != 0)
    require(c.architecture == kSharedNeighbor || c.architecture == kFullMesh,
            "only a full mesh configures its mesh initialization");
  if (c.architecture == kFullMesh)
    require(c.encoding == kBinary && c.connectivity != kOwn,
            "a full mesh needs ordinary binary inputs and two-parent connectivity");
  if (c.architecture == kSharedNeighbor)
    require(c.width >= c.modulus && c.width % 2 == 0 && c.connectivity != kOwn,
            "shared Neighbor meshes need one-hot inputs, even width >= classes, two core parents and "
            "embedding depth 1..=64");
  require(c.mesh_learning_rate_multiplier >= 1, "the mesh learning rate multiplier must be positive");
  if (c.mesh_learning_rate_multiplier != 1)
    require(mesh_layers(c) > 0, "only mesh layers multiply their learning rate");
  require(parameter_count(c) <= kMaxParameters, "models are limited to 268435456 parameters");
}

void validate_kernel_shapes(const mb_simple_config& c) {
  validate(c);
  require(c.width <= kMaxKernelWidth, "this build's fused row kernels support widths up to 512", MB_ERR_UNSUPPORTED);
  if (c.architecture == kFullMesh)
    require(c.width <= 256 && c.modulus <= 256, "this build's full mesh kernels support widths and moduli up to 256",
            MB_ERR_UNSUPPORTED);
}

namespace {
struct Normal {
  double radius, angle;
};
Normal box_muller(Random& r) {
  const double radius = std::sqrt(-2.0 * std::log(1.0 - (double)r.unit()));
  const double angle = 6.283185307179586 * (double)r.unit();  // TAU
  return {radius, angle};
}
}  // namespace

std::vector<float> initial_parameters(const mb_simple_config& c, uint64_t seed) {
  validate(c);
  Random r(seed ^ 0x73696d706c650004ull);
  std::vector<float> p;
  p.reserve(parameter_count(c));
  const uint32_t w = c.width;
  if (c.architecture == kSharedNeighbor) {
    const double ratio = 0.1 / std::sqrt((double)c.embedding_mesh_depth);  // near-identity
    const double deviation = ratio * 1.0;
    for (size_t i = 0; i < (size_t)c.embedding_mesh_depth * w; ++i) {
      const Normal n = box_muller(r);
      p.push_back(1.0f);
      p.push_back((float)(deviation * n.radius * std::cos(n.angle)));
    }
    for (uint32_t layer = 0; layer < c.depth; ++layer) {
      const bool identity = c.full_mesh_initialization == 1 && layer > 0;
      for (uint32_t u = 0; u < w; ++u) {
        if (identity) {
          p.push_back(1.0f);
          p.push_back(0.0f);
        } else {
          const Normal n = box_muller(r);
          p.push_back((float)(n.radius * std::cos(n.angle)));
          p.push_back((float)(n.radius * std::sin(n.angle)));
        }
        p.push_back(0.0f);
      }
    }
    return p;
  }
  if (c.architecture == kFullMesh) {
    // src/simple/mod.rs:979-1003: Box-Muller pairs (deviation sqrt(1/2) on
    // the readout), identity hidden layers on request, zero biases.
    const auto tl = two_parent_layers(c);
    for (size_t index = 0; index < tl.size(); ++index) {
      const bool identity = c.full_mesh_initialization == 1 && index > 0 && index < c.depth;
      const double deviation = index == c.depth ? std::sqrt(0.5) : 1.0;
      for (uint32_t u = 0; u < tl[index].outputs; ++u) {
        if (identity) {
          p.push_back(1.0f);
          p.push_back(0.0f);
        } else {
          const Normal n = box_muller(r);
          p.push_back((float)(deviation * n.radius * std::cos(n.angle)));
          p.push_back((float)(deviation * n.radius * std::sin(n.angle)));
        }
        p.push_back(0.0f);
      }
    }
    return p;
  }
  const auto layers = dense_layers(c);
  for (size_t index = 0; index < layers.size(); ++index) {
    const size_t count = (size_t)layers[index].first * layers[index].second;
    if (c.architecture == kRotaryDense && index > 0) {
      const double deviation = std::sqrt(2.0 / (double)layers[index].first);  // Kaiming normal, ReLU gain
      for (size_t off = 0; off < count; off += 2) {
        const Normal n = box_muller(r);
        p.push_back((float)(deviation * n.radius * std::cos(n.angle)));
        if (off + 1 < count) p.push_back((float)(deviation * n.radius * std::sin(n.angle)));
      }
      continue;
    }
    const float bound = 1.0f / std::sqrt((float)layers[index].first);
    for (size_t i = 0; i < count; ++i) p.push_back((2.0f * r.unit() - 1.0f) * bound);
  }
  for (size_t i = 0; i < (size_t)stored_mesh_layers(c) * w; ++i) {
    p.push_back(1.0f);
    if (parents(c) == 2) p.push_back(0.0f);
  }
  return p;
}

void decode_operands(const mb_simple_config& c, const float* features, const uint32_t* targets, size_t rows,
                     std::vector<uint32_t>& a, std::vector<uint32_t>& b) {
  const uint32_t m = c.modulus, f = operand_features(c);
  const std::vector<float> table = encoding_table(c);
  a.resize(rows);
  b.resize(rows);
  for (size_t r = 0; r < rows; ++r) {
    require(targets[r] < m, "answer classes must be below the modulus");
    for (int half = 0; half < 2; ++half) {
      const float* x = features + r * 2 * f + half * f;
      for (uint32_t k = 0; k < f; ++k)
        require(std::isfinite(x[k]), "features must contain only finite values", MB_ERR_NONFINITE);
      uint32_t hit = m;
      if (c.encoding == kOneHot) {
        for (uint32_t k = 0; k < m; ++k) {
          if (x[k] == 1.0f && hit == m) {
            hit = k;
          } else {
            require(x[k] == 0.0f, "this build's kernels read encoded operand rows", MB_ERR_UNSUPPORTED);
          }
        }
      } else {
        for (uint32_t v = 0; v < m && hit == m; ++v)
          if (std::memcmp(x, table.data() + (size_t)v * f, f * sizeof(float)) == 0) hit = v;
      }
      require(hit < m, "this build's kernels read encoded operand rows", MB_ERR_UNSUPPORTED);
      (half == 0 ? a : b)[r] = hit;
    }
  }
}

}  // namespace simple
}  // namespace mb
