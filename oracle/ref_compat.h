/*
 * Test infrastructure only (oracle).  Force-included (g++ -include) when the
 * reference's asdsl/kernels/native/gemv_q4_avx2.cpp is compiled from its own
 * source tree into oracle/_ref/.
 *
 * That translation unit defines a global `inline float _cvtsh_ss(unsigned short)`
 * (asdsl/kernels/native/gemv_q4_avx2.cpp:1510), which collides with GCC's
 * F16C intrinsic of the same name and is a hard error under g++.  Every use of
 * the name in that file comes after its definition, so renaming the token for
 * that one TU (after the intrinsic headers have been seen once) lets the file
 * compile unmodified; its own definition then serves its own calls.
 */
#pragma once
#include <immintrin.h>
#define _cvtsh_ss asdsl_ref_cvtsh_ss_local
