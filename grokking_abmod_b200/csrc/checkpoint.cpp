// Mesh GPT weight checkpoints in the reference's MSHGPT07 / MSHGPT08 layouts
// (src/gpt/checkpoint.rs:25-196): an 8-byte magic, the configuration as
// little-endian u32 fields, the tokenizer's characters as u32 code points
// and the parameters as little-endian f32, with nothing after them.
// MSHGPT07 is the default architecture (mesh token embedding, Neighbor
// connectivity); MSHGPT08 adds the (embedding, connectivity) fields.  The
// MSHGPT09 geometry ablations are outside this build's kernels and load as
// MB_ERR_UNSUPPORTED.  Loading a checkpoint into a model
// goes through set_parameters, which resets AdamW as the reference's loader
// does.

#include <cmath>
#include <cstdio>
#include <cstring>
#include <set>
#include <string>
#include <vector>

#include "host.h"

namespace mb {

namespace {

constexpr size_t kMaxVocab = 65536;  // src/gpt/mod.rs (MODEL_MAX_VOCAB)

bool valid_char(uint32_t c) { return c <= 0x10FFFF && !(c >= 0xD800 && c <= 0xDFFF); }

void validate_characters(const uint32_t* chars, size_t n) {
  // CharacterTokenizer::from_characters (src/gpt/text.rs:17-24)
  require(n >= 2 && n <= kMaxVocab, "tokenizer must contain 2..65536 unique characters");
  std::set<uint32_t> seen;
  for (size_t i = 0; i < n; ++i) {
    require(valid_char(chars[i]), "invalid checkpoint character");
    seen.insert(chars[i]);
  }
  require(seen.size() == n, "tokenizer must contain 2..65536 unique characters");
}

void put_u32(std::vector<unsigned char>& out, uint32_t v) {
  for (int i = 0; i < 4; ++i) out.push_back((unsigned char)(v >> (8 * i)));
}

uint32_t get_u32(const std::vector<unsigned char>& in, size_t& pos) {
  require(pos + 4 <= in.size(), "checkpoint is truncated");
  uint32_t v = 0;
  for (int i = 0; i < 4; ++i) v |= (uint32_t)in[pos + i] << (8 * i);
  pos += 4;
  return v;
}

}  // namespace

void write_checkpoint(const std::string& path, const mb_gpt_config& c, const uint32_t* chars, size_t n_chars,
                      const float* params, size_t n_params) {
  validate_config(c);
  require(make_layout(c).count() == n_params && c.vocab_size == n_chars,
          "checkpoint model, parameters, and tokenizer do not match");
  validate_characters(chars, n_chars);
  for (size_t i = 0; i < n_params; ++i)
    require(std::isfinite(params[i]), "checkpoint parameters must be finite", MB_ERR_NONFINITE);
  const bool default_layout = c.connectivity == 0 && c.embedding == 0;
  std::vector<unsigned char> out;
  out.reserve(8 + 4 * (9 + n_chars + n_params));
  const char* magic = default_layout ? "MSHGPT07" : "MSHGPT08";
  out.insert(out.end(), magic, magic + 8);
  for (uint32_t f : {c.vocab_size, c.context, c.width, c.heads, c.layers, c.attention_mesh_depth, c.ffn_mesh_depth})
    put_u32(out, f);
  if (!default_layout) {
    put_u32(out, c.embedding);
    put_u32(out, c.connectivity);
  }
  for (size_t i = 0; i < n_chars; ++i) put_u32(out, chars[i]);
  for (size_t i = 0; i < n_params; ++i) {
    uint32_t bits;
    std::memcpy(&bits, params + i, 4);
    put_u32(out, bits);
  }
  FILE* f = std::fopen(path.c_str(), "wb");
  require(f != nullptr, "cannot create checkpoint file: " + path);
  const size_t wrote = std::fwrite(out.data(), 1, out.size(), f);
  const int closed = std::fclose(f);
  require(wrote == out.size() && closed == 0, "cannot write checkpoint file: " + path);
}

void read_checkpoint(const std::string& path, mb_gpt_config& c, std::vector<uint32_t>& chars,
                     std::vector<float>& params) {
  FILE* f = std::fopen(path.c_str(), "rb");
  require(f != nullptr, "cannot open checkpoint file: " + path);
  std::vector<unsigned char> in;
  unsigned char buf[1 << 16];
  size_t got;
  while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) in.insert(in.end(), buf, buf + got);
  std::fclose(f);
  require(in.size() >= 8, "unsupported Mesh GPT checkpoint format");
  const std::string magic(reinterpret_cast<const char*>(in.data()), 8);
  if (magic != "MSHGPT07" && magic != "MSHGPT08" && magic != "MSHGPT09") {
    if (magic == "MSHGPT01" || magic == "MSHGPT02")
      throw Error(MB_ERR_INVALID, "checkpoint uses learned position embeddings; retrain Mesh GPT with RoPE");
    if (magic == "MSHGPT03") throw Error(MB_ERR_INVALID, "checkpoint uses LayerNorm; retrain Mesh GPT with RMSNorm");
    if (magic == "MSHGPT04") throw Error(MB_ERR_INVALID, "checkpoint contains biases; retrain bias-free Mesh GPT");
    if (magic == "MSHGPT05")
      throw Error(MB_ERR_INVALID,
                  "checkpoint uses learned RMSNorm without QK-Norm; retrain Mesh GPT with parameter-free QK-Norm");
    if (magic == "MSHGPT06")
      throw Error(MB_ERR_INVALID,
                  "checkpoint uses a learned token table; retrain Mesh GPT with mesh token embeddings");
    throw Error(MB_ERR_INVALID, "unsupported Mesh GPT checkpoint format");
  }
  require(magic != "MSHGPT09", "MSHGPT09 geometry ablations are outside this build", MB_ERR_UNSUPPORTED);
  size_t pos = 8;
  c.vocab_size = get_u32(in, pos);
  c.context = get_u32(in, pos);
  c.width = get_u32(in, pos);
  c.heads = get_u32(in, pos);
  c.layers = get_u32(in, pos);
  c.attention_mesh_depth = get_u32(in, pos);
  c.ffn_mesh_depth = get_u32(in, pos);
  c.connectivity = 0;
  c.embedding = 0;
  if (magic == "MSHGPT08") {
    const uint32_t embedding = get_u32(in, pos);
    const uint32_t connectivity = get_u32(in, pos);
    require(embedding <= 1, "unknown checkpoint token embedding");
    require(connectivity <= 1, "unknown checkpoint mesh connectivity");
    require(!(embedding == 0 && connectivity == 0), "the default architecture must use the MSHGPT07 layout");
    c.embedding = embedding;
    c.connectivity = connectivity;
  }
  validate_config(c);
  const size_t count = make_layout(c).count();
  chars.resize(c.vocab_size);
  for (auto& ch : chars) ch = get_u32(in, pos);
  validate_characters(chars.data(), chars.size());
  params.resize(count);
  for (auto& p : params) {
    const uint32_t bits = get_u32(in, pos);
    std::memcpy(&p, &bits, 4);
    require(std::isfinite(p), "checkpoint parameters must be finite", MB_ERR_NONFINITE);
  }
  require(pos == in.size(), "unexpected trailing checkpoint bytes");
}

}  // namespace mb

extern "C" {

int mb_gpt_checkpoint_write(const char* path, const mb_gpt_config* config, const uint32_t* characters,
                            size_t n_characters, const float* parameters, size_t n_parameters) {
  return mb::guarded([&] {
    mb::need(path, "path");
    mb::need(config, "config");
    mb::need(characters, "characters");
    mb::need(parameters, "parameters");
    mb::write_checkpoint(path, *config, characters, n_characters, parameters, n_parameters);
  });
}

int mb_gpt_checkpoint_read(const char* path, mb_gpt_config* config, uint32_t* characters, size_t* n_characters,
                           float* parameters, size_t* n_parameters) {
  return mb::guarded([&] {
    mb::need(path, "path");
    mb::need(config, "config");
    mb::need(n_characters, "n_characters");
    mb::need(n_parameters, "n_parameters");
    std::vector<uint32_t> chars;
    std::vector<float> params;
    mb::read_checkpoint(path, *config, chars, params);
    if (characters != nullptr) {
      mb::require(*n_characters >= chars.size(), "characters buffer is too small");
      std::memcpy(characters, chars.data(), chars.size() * 4);
    }
    if (parameters != nullptr) {
      mb::require(*n_parameters >= params.size(), "parameters buffer is too small");
      std::memcpy(parameters, params.data(), params.size() * 4);
    }
    *n_characters = chars.size();
    *n_parameters = params.size();
  });
}

}  // extern "C"
