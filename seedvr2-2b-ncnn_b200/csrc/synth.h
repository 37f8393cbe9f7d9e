// synth.h -- seeded synthetic weights/inputs (Philox4x32-10 + Box-Muller).
#pragma once
#include "s2b_common.h"
#include <string>
#include <vector>

namespace s2b {

constexpr float SYNTH_STD = 0.02f;   // weights N(0, 0.02); scales/gates/norm weights 1 + N(0, 0.02)

struct SynthLinear { std::string name; int out, in; bool has_bias; };
struct SynthVector { std::string name; int n; float mean; };

void philox4x32_10(const uint32_t ctr[4], uint64_t seed, uint32_t out[4]);
void fill_normal_f32(float* out, size_t n, uint64_t seed, uint64_t stream, float mean, float stdv);
void fill_normal_f16(uint16_t* out, size_t n, uint64_t seed, uint64_t stream, float mean, float stdv);
uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);

// Linear layers present for layers [layer_lo, layer_hi) plus the top-level ones.
std::vector<SynthLinear> model_linears(int layer_lo, int layer_hi);
// Every raw fp32 vector the model needs (all 32 layers' norm/ada branches).
std::vector<SynthVector> model_vectors();
void synth_linear(const SynthLinear& L, uint64_t seed, uint16_t* w_f16, float* bias);
void synth_vector(const SynthVector& V, uint64_t seed, float* out);
int write_m5(const char* dir, uint64_t seed, int layer_lo, int layer_hi, std::string& err);

void synth_vid_grid(float* grid, int T, int H, int W, uint64_t seed);
void synth_txt(float* txt, int TXT, uint64_t seed);

}  // namespace s2b
