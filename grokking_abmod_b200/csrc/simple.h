// grok-simple models: host configuration, layout and initialisation shared
// by the executor (simple_model.cu) and the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "host.h"

namespace mb {
namespace simple {

enum Architecture : uint32_t { kMeshMlp = 0, kRotaryDense = 1, kSharedNeighbor = 2, kMlp = 3, kBilinear = 4,
                               kResidualMlp = 5, kResidualMesh = 6, kTiedConcatResidualMesh = 7,
                               kTiedRotaryResidualMesh = 8, kTiedConcatMesh = 9, kFullMesh = 10 };
enum Activation : uint32_t { kRelu = 0, kSquare = 1 };
enum Encoding : uint32_t { kOneHot = 0, kBinary = 1, kScalar = 2, kDiscreteLog = 3 };
enum Connectivity : uint32_t { kOwn = 0, kNeighbor = 1, kButterfly = 2 };

constexpr uint32_t kMaxWidth = 16384, kMaxDepth = 64, kMaxClasses = 1024;  // src/simple/mod.rs:25-31
constexpr size_t kMaxRows = 131072;
constexpr size_t kMaxParameters = (size_t)1 << 28;
// This build's fused row kernels keep a row per warp in shared memory.
constexpr uint32_t kMaxKernelWidth = 512;

// src/simple/mod.rs:113-147
inline bool residual_mesh(const mb_simple_config& c) {
  return c.architecture == kResidualMesh || c.architecture == kTiedConcatResidualMesh ||
         c.architecture == kTiedRotaryResidualMesh;
}
inline bool tied_concat(const mb_simple_config& c) {
  return c.architecture == kTiedConcatResidualMesh || c.architecture == kTiedConcatMesh;
}

void validate(const mb_simple_config& c);                // the reference's rules (MB_ERR_INVALID)
void validate_kernel_shapes(const mb_simple_config& c);  // this build's kernels (MB_ERR_UNSUPPORTED)
int parents(const mb_simple_config& c);
int stride(const mb_simple_config& c, int layer);
int mesh_layers(const mb_simple_config& c);
// Mesh layers with their own weights: at most one when they are tied
// (src/simple/mod.rs:880-893).
int stored_mesh_layers(const mb_simple_config& c);
// A full mesh layer: unit o reads inputs o * inputs / outputs and that plus
// stride (mod inputs) (TwoParentLayer, src/simple/mod.rs:486-501).
struct TwoParentLayer {
  uint32_t inputs, outputs, stride;
};
// The full mesh's layers, input layer to readout (src/simple/mod.rs:766-800).
std::vector<TwoParentLayer> two_parent_layers(const mb_simple_config& c);
// Dense (inputs, outputs) layers in parameter order.
std::vector<std::pair<uint32_t, uint32_t>> dense_layers(const mb_simple_config& c);
std::vector<size_t> groups(const mb_simple_config& c);
size_t parameter_count(const mb_simple_config& c);
std::vector<float> initial_parameters(const mb_simple_config& c, uint64_t seed);
// Features per operand (Encoding::features, src/simple/mod.rs:362-370).
uint32_t operand_features(const mb_simple_config& c);
// One feature row per residue, [modulus][operand_features]
// (Encoding::table, src/simple/mod.rs:373-414).
std::vector<float> encoding_table(const mb_simple_config& c);
// Encoded rows -> operand residues: each operand block must equal one row
// of the encoding table (MB_ERR_UNSUPPORTED otherwise).
void decode_operands(const mb_simple_config& c, const float* features, const uint32_t* targets, size_t rows,
                     std::vector<uint32_t>& a, std::vector<uint32_t>& b);

}  // namespace simple
}  // namespace mb
