// Device-side synthetic checkpoint generator (see synth.cu).
#pragma once

#include <algorithm>
#include <string>

#include "common.h"

namespace swl {

enum SynthRole : int { SYN_NORM = 1, SYN_ALOG = 2, SYN_DTBIAS = 3, SYN_CONV = 4, SYN_OTHER = 5 };

uint64_t synth_key(const std::string& name, uint64_t seed);
// Packed uint32 words of `name`; element i goes to dense dst[i] (pe == 0) or
// to blob (i / pe) at dst + (i / pe) * stride + (i % pe) * 4.
void synth_words(uint8_t* dst, const std::string& name, uint64_t seed, int64_t n, int64_t pe, int64_t stride, cudaStream_t st);
// Scales and biases of quantised module `module` (same placement rule).
void synth_affine(uint8_t* ds, uint8_t* db, const std::string& module, uint64_t seed, int bits, float wstd, bool bf16,
                  int64_t n, int64_t pe, int64_t stride, cudaStream_t st);
// A plain tensor written as f32 values (bf16-rounded when the synthetic
// checkpoint stores it as bf16).
void synth_plain(float* dst, const std::string& name, uint64_t seed, int role, float wstd, bool bf16, int64_t n, cudaStream_t st);

}  // namespace swl
