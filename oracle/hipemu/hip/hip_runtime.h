// CPU stand-in for <hip/hip_runtime.h> — TEST INFRASTRUCTURE ONLY.
// The reference's kernel sources include this header; it brings in the types and runtime of hipemu_core.h and maps
// the HIP dialect (qualifiers, thread indices, builtins) onto them. See hipemu_core.h for what each stand-in does
// and how it differs from the gfx1030 hardware.
#pragma once
#include "../hipemu_core.h"

// ---------------------------------------------------------------- keywords and builtins of the HIP dialect
#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __shared__ thread_local
#define threadIdx (::hipemu::thread_index())
#define blockIdx (::hipemu::block_index)
#define blockDim (::hipemu::block_dim)
#define gridDim (::hipemu::grid_dim)
#define __syncthreads() ::hipemu::block_barrier()
#define __shfl_xor(v, m, w) ::hipemu::shfl_xor((v), (m), (w))
#define __any(p) ::hipemu::any(p)
#define __builtin_shufflevector(a, b, ...) ::hipemu::shufflevector((a), (b), __VA_ARGS__)
#define __builtin_nontemporal_load(p) (*(p))
#define __builtin_amdgcn_readfirstlane(x) (x)
#define __builtin_amdgcn_sched_barrier(x) ((void)0)
#define __builtin_amdgcn_fence(...) ((void)0)
#define __builtin_amdgcn_s_barrier() ::hipemu::block_barrier()
#define __builtin_amdgcn_wave_barrier() ::hipemu::wave_barrier()
#define __builtin_amdgcn_sdot4(a, b, c, clamp) ::hipemu::sdot4((a), (b), (c), (clamp))
#define __builtin_amdgcn_sdot8(a, b, c, clamp) ::hipemu::sdot8((a), (b), (c), (clamp))
#define __builtin_amdgcn_fdot2(a, b, c, clamp) ::hipemu::fdot2((a), (b), (c), (clamp))
#define __builtin_amdgcn_exp2f(x) exp2f(x)
// Inline assembly in the kernels only pins values to registers (scheduling hints); it has no effect here.
#define asm
#define volatile(...) ((void)0)
