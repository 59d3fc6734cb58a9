// CPU stand-in for the HIP device environment: types and runtime interface — TEST INFRASTRUCTURE ONLY.
//
// It lets g++ compile the reference's own kernel sources (int8_gemm.hip, hip_attention.hip, int8_gemv.hip,
// rms_norm.hip) unmodified apart from their vector typedefs (see oracle/hipemu/build.py), and run them on the host:
// every GPU thread of a block is a fiber on one OS thread, blocks run on a pool of OS threads, __shared__ arrays are
// per-OS-thread statics (so a block's fibers share them), and the synchronising operations the kernels use
// (__syncthreads, s_barrier, wave barriers, __shfl_xor, __any) are rendezvous points of the block's or the wave's
// fibers. Waves are 32 lanes wide (the reference's kernels index lanes as threadIdx.x & 31).
//
// Arithmetic stand-ins, and how they differ from the gfx1030 hardware (the tests that use this oracle state a
// tolerance wherever one of these is on the path):
//   sdot4 / sdot8           exact integer dot products (the hardware's are exact too)
//   fdot2                   a.x*b.x + a.y*b.y + c with the fp16 products exact and one rounding of the sum
//   exp2f (amdgcn), expf    the C library's, correctly rounded or within 1 ulp (the hardware's are ~1 ulp)
//   rsqrtf                  1 / sqrtf, both correctly rounded (the hardware's v_rsq is ~1 ulp)
//   floating-point contraction is off (-ffp-contract=off); the reference's compiler contracts a multiply-add
//   outside the regions where its source switches contraction off.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <functional>
#include <type_traits>
#include <utility>

namespace hipemu {

struct Dim3 {
    unsigned x, y, z;
};

// The fiber of the GPU thread being run on this OS thread.
struct Fiber;
extern thread_local Fiber* current;
extern thread_local Dim3 block_index, block_dim, grid_dim;
const Dim3& thread_index();
int lane_of_current();
int wave_of_current();

void block_barrier();
void wave_barrier();
// Runs `kernel` once per GPU thread of every block of the grid (blocks in parallel on host threads); returns when
// all have finished.
void launch(Dim3 grid, Dim3 block, const std::function<void()>& kernel);
// Publishes this lane's 64-bit value and returns the wave's table of them (valid until the next wave barrier).
const uint64_t* wave_exchange(uint64_t mine);

// ---------------------------------------------------------------- vector types (clang ext_vector_type)
#define HIPEMU_VEC_OPS(N)                                                                  \
    T& operator[](int i) { return v[i]; }                                                  \
    const T& operator[](int i) const { return v[i]; }                                      \
    Vec operator*(const Vec& o) const {                                                    \
        Vec r;                                                                             \
        for (int i = 0; i < N; ++i) r.v[i] = v[i] * o.v[i];                                \
        return r;                                                                          \
    }                                                                                      \
    Vec operator+(const Vec& o) const {                                                    \
        Vec r;                                                                             \
        for (int i = 0; i < N; ++i) r.v[i] = v[i] + o.v[i];                                \
        return r;                                                                          \
    }                                                                                      \
    Vec operator*(T s) const {                                                             \
        Vec r;                                                                             \
        for (int i = 0; i < N; ++i) r.v[i] = v[i] * s;                                     \
        return r;                                                                          \
    }

template <class T, int N>
struct Vec {
    T v[N];
    HIPEMU_VEC_OPS(N)
};
template <class T>
struct Vec<T, 2> {
    union {
        T v[2];
        struct {
            T x, y;
        };
    };
    HIPEMU_VEC_OPS(2)
};
template <class T>
struct Vec<T, 4> {
    union {
        T v[4];
        struct {
            T x, y, z, w;
        };
    };
    HIPEMU_VEC_OPS(4)
};

template <class T, int N, class... I>
Vec<T, (int)sizeof...(I)> shufflevector(const Vec<T, N>& a, const Vec<T, N>& b, I... idx) {
    Vec<T, (int)sizeof...(I)> r;
    const int ids[] = {(int)idx...};
    for (int i = 0; i < (int)sizeof...(I); ++i) r.v[i] = ids[i] < N ? a.v[ids[i]] : b.v[ids[i] - N];
    return r;
}

// ---------------------------------------------------------------- cross-lane operations
template <class T>
T shfl_xor(T value, int mask, int width) {
    static_assert(sizeof(T) <= 8 && std::is_trivially_copyable<T>::value, "shuffle of a register-sized value");
    uint64_t bits = 0;
    memcpy(&bits, &value, sizeof(T));
    const uint64_t* all = wave_exchange(bits);
    const int lane = lane_of_current();
    const int src = (lane & ~(width - 1)) | ((lane ^ mask) & (width - 1));
    T r;
    memcpy(&r, &all[src], sizeof(T));
    wave_barrier();  // nobody overwrites the table before every lane has read it
    return r;
}
bool any(bool p);

// ---------------------------------------------------------------- amdgcn builtins
inline int sdot4(int a, int b, int c, bool) {
    int acc = c;
    for (int i = 0; i < 4; ++i) acc += (int)(int8_t)(a >> (8 * i)) * (int)(int8_t)(b >> (8 * i));
    return acc;
}
inline int sdot8(int a, int b, int c, bool) {
    int acc = c;
    for (int i = 0; i < 8; ++i) {
        const int x = (int)((uint32_t)a << (28 - 4 * i)) >> 28, y = (int)((uint32_t)b << (28 - 4 * i)) >> 28;
        acc += x * y;
    }
    return acc;
}
template <class H2>
inline float fdot2(H2 a, H2 b, float c, bool) {
    // fp16 x fp16 products are exact in float; the sum of the three terms is rounded once (through double, where
    // the two exact products and c add without rounding in all but far-apart exponent cases).
    const double s = (double)((float)a.v[0] * (float)b.v[0]) + (double)((float)a.v[1] * (float)b.v[1]) + (double)c;
    return (float)s;
}

}  // namespace hipemu

inline float rsqrtf(float x) { return 1.0f / sqrtf(x); }
inline int min(int a, int b) { return a < b ? a : b; }
inline int max(int a, int b) { return a > b ? a : b; }

