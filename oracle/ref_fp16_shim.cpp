// TEST INFRASTRUCTURE ONLY. Exposes the reference's host FP16 converter
// (native/fp16.hpp:11-44, included from the reference tree at build time) as a
// C symbol so tests can compare this repository's converters against it.
#include "fp16.hpp"
extern "C" unsigned short ref_to_fp16(float value) { return jade::to_fp16(value); }
