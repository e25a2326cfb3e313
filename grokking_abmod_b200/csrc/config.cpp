// Mesh GPT configuration, parameter layout, seeded initialisation, token codes
// and batch validation (host side of the C ABI).
//
// Restates src/gpt/config.rs: validation :144-172, strides :117-122, Layout
// :358-414, Layout::initialize :416-459 (mesh embedding, default geometry),
// token_codes :552-591, validate_tokens/validate_batch :210-253 and
// AdamWOptions::validate :279-295.  Compiled with -ffp-contract=off so the
// f32 initialisation arithmetic rounds exactly like the reference.

#include <cmath>
#include <string>

#include "host.h"

namespace mb {

namespace {
constexpr size_t kMaxRows = 131072;  // src/gpt/mod.rs:30
}

void validate_config(const mb_gpt_config& c) {
  require(c.vocab_size >= 2 && c.vocab_size <= 65536, "vocab_size must be in 2..65536");
  require(c.context >= 1 && c.context <= 4096, "context must be in 1..4096");
  require(c.width >= 2 && c.width <= 4096, "width must be in 2..4096");
  require(c.heads >= 1 && c.heads <= 64 && c.width % c.heads == 0, "heads must be in 1..64 and divide width");
  require(c.width / c.heads >= 2, "each attention head requires at least two channels");
  require((c.width / c.heads) % 2 == 0, "slice RoPE requires an even number of channels per head");
  require(c.layers >= 1 && c.layers <= 64, "layers must be in 1..64");
  require(c.attention_mesh_depth >= 1 && c.attention_mesh_depth <= 256 && c.ffn_mesh_depth >= 1 &&
              c.ffn_mesh_depth <= 256,
          "mesh depths must be in 1..256");
  require(c.connectivity <= 1, "connectivity must be 0 (neighbor) or 1 (butterfly)");
  require(c.embedding <= 1, "embedding must be 0 (mesh) or 1 (table)");
}

void validate_kernel_shapes(const mb_gpt_config& c) {
  validate_config(c);
  const uint32_t hd = c.width / c.heads;
  const bool width_ok = c.width == 64 || c.width == 128 || c.width == 256 || c.width == 384 || c.width == 512;
  require(width_ok, "this build's fused kernels support widths 64, 128, 256, 384 and 512", MB_ERR_UNSUPPORTED);
  require(hd <= 128 && (hd & (hd - 1)) == 0, "this build's kernels support power-of-two head widths up to 128",
          MB_ERR_UNSUPPORTED);
  require((size_t)c.vocab_size * c.width <= 65536 && c.vocab_size <= 1024,
          "this build's fused head supports vocab * width <= 65536", MB_ERR_UNSUPPORTED);
  require(c.attention_mesh_depth <= 16 && c.ffn_mesh_depth <= 16,
          "this build's fused block kernels support mesh depths up to 16", MB_ERR_UNSUPPORTED);
}

int mesh_stride(const mb_gpt_config& c, int layer) {
  if (c.connectivity == 0) return 1;
  int log2w = 31 - __builtin_clz(c.width);
  return 1 << (layer % log2w);
}

Layout make_layout(const mb_gpt_config& c) {
  validate_config(c);
  Layout l;
  auto push = [&](size_t size, int depth) {
    l.groups.push_back(Group{l.count(), size, depth});
    return (int)l.groups.size() - 1;
  };
  const size_t w = c.width;
  // A table has no mesh layers (src/gpt/config.rs:366-372).
  l.embedding = c.embedding == 0 ? push(2 * w * c.attention_mesh_depth, c.attention_mesh_depth)
                                 : push((size_t)c.vocab_size * w, 0);
  for (uint32_t b = 0; b < c.layers; ++b) {
    BlockGroups g;
    g.query = push(2 * w * c.attention_mesh_depth, c.attention_mesh_depth);
    g.key = push(2 * w * c.attention_mesh_depth, c.attention_mesh_depth);
    g.value = push(2 * w * c.attention_mesh_depth, c.attention_mesh_depth);
    g.projection = push(2 * w * c.attention_mesh_depth, c.attention_mesh_depth);
    g.ffn = push(2 * w * c.ffn_mesh_depth, c.ffn_mesh_depth);
    l.blocks.push_back(g);
  }
  return l;
}

std::vector<float> tabulated(const mb_gpt_config& mesh, const std::vector<float>& params);

std::vector<float> initial_parameters(const mb_gpt_config& c, uint64_t seed) {
  if (c.embedding == 1) {
    // A table draws the mesh model's stream and stores its tabulated
    // embedding, so both start as one function (src/gpt/config.rs:416-433).
    mb_gpt_config mesh = c;
    mesh.embedding = 0;
    return tabulated(mesh, initial_parameters(mesh, seed));
  }
  const Layout layout = make_layout(c);
  Random random(seed);
  std::vector<float> p(layout.count(), 0.0f);
  for (const Group& g : layout.groups) {
    for (int layer = 0; layer < g.depth; ++layer) {
      for (uint32_t ch = 0; ch < c.width; ++ch) {
        const size_t o = g.offset + (size_t)layer * 2 * c.width + (size_t)ch * 2;
        float a = 0.7f + 0.2f * (random.unit() - 0.5f);
        float b = 0.4f * (random.unit() - 0.5f);
        if (layer + 1 == g.depth) {
          a *= 0.3f;
          b *= 0.3f;
        }
        p[o] = a;
        p[o + 1] = b;
      }
    }
  }
  return p;
}

// The mesh embedding of every token code in f64 (ELU through expm1), cast to
// f32, followed by the block parameters (src/gpt/config.rs:515-546).
std::vector<float> tabulated(const mb_gpt_config& mesh, const std::vector<float>& params) {
  const uint32_t v = mesh.vocab_size, w = mesh.width, depth = mesh.attention_mesh_depth;
  const std::vector<float> codes = token_codes(mesh);
  std::vector<double> cur(codes.begin(), codes.end()), next((size_t)v * w);
  for (uint32_t layer = 0; layer < depth; ++layer) {
    const uint32_t stride = (uint32_t)mesh_stride(mesh, (int)layer);
    for (uint32_t t = 0; t < v; ++t) {
      const double* in = cur.data() + (size_t)t * w;
      for (uint32_t ch = 0; ch < w; ++ch) {
        const size_t p = (size_t)layer * 2 * w + 2 * ch;
        const double sum = in[ch] * (double)params[p] + in[(ch + stride) % w] * (double)params[p + 1];
        next[(size_t)t * w + ch] = layer + 1 != depth && sum < 0.0 ? std::expm1(sum) : sum;
      }
    }
    cur.swap(next);
  }
  std::vector<float> out;
  out.reserve((size_t)v * w + params.size() - (size_t)2 * w * depth);
  for (double x : cur) out.push_back((float)x);
  out.insert(out.end(), params.begin() + (size_t)2 * w * depth, params.end());
  return out;
}

std::vector<float> token_codes(const mb_gpt_config& c) {
  validate_config(c);
  const uint32_t v = c.vocab_size, w = c.width;
  const uint32_t bits = 32 - __builtin_clz(v - 1);
  const uint32_t lanes = w < bits ? w : bits;
  std::vector<uint32_t> masks;
  for (uint32_t b = 0; b < bits; ++b) masks.push_back(1u << b);
  for (uint32_t m = 1; m < (1u << bits); ++m)
    if (m & (m - 1)) masks.push_back(m);
  std::vector<float> codes((size_t)v * w);
  for (uint32_t t = 0; t < v; ++t) {
    for (uint32_t ch = 0; ch < w; ++ch) {
      float value;
      if (w >= bits) {
        value = (__builtin_popcount(t & masks[ch % masks.size()]) % 2 == 0) ? -1.0f : 1.0f;
      } else {
        uint32_t digit = 0, maximum = 0;
        for (uint32_t bit = ch % lanes; bit < bits; bit += lanes) {
          digit = 2 * digit + ((t >> bit) & 1);
          maximum = 2 * maximum + 1;
        }
        value = 2.0f * (float)digit / (float)maximum - 1.0f;
      }
      codes[(size_t)t * w + ch] = value;
    }
  }
  return codes;
}

size_t validate_batch(const mb_gpt_config& c, const uint32_t* inputs, const uint32_t* targets, size_t rows,
                      size_t sequence, bool allow_unsupervised) {
  require(sequence >= 1 && sequence <= c.context && rows >= 1 && rows % sequence == 0 && rows <= kMaxRows,
          "tokens must form a nonempty batch of equal sequences within context and 131072 rows");
  require(inputs != nullptr, "inputs must not be null");
  for (size_t i = 0; i < rows; ++i) require(inputs[i] < c.vocab_size, "token ID is outside the vocabulary");
  if (targets == nullptr) return 0;
  size_t supervised = 0;
  for (size_t i = 0; i < rows; ++i) {
    if (targets[i] != MB_IGNORE_TARGET) {
      require(targets[i] < c.vocab_size, "target ID is outside the vocabulary");
      ++supervised;
    }
  }
  require(supervised > 0 || allow_unsupervised, "batch must contain at least one supervised target");
  return supervised;
}

void validate_optimizer(const mb_adamw& o) {
  const bool ok = std::isfinite(o.learning_rate) && o.learning_rate > 0.0f && std::isfinite(o.weight_decay) &&
                  o.weight_decay >= 0.0f && std::isfinite(o.beta1) && o.beta1 >= 0.0f && o.beta1 < 1.0f &&
                  std::isfinite(o.beta2) && o.beta2 >= 0.0f && o.beta2 < 1.0f && std::isfinite(o.epsilon) &&
                  o.epsilon > 0.0f;
  require(ok,
          "AdamW requires finite positive learning rate/epsilon, nonnegative decay, and betas in [0, 1)");
}

}  // namespace mb
