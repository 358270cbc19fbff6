// Shared device helpers for the batmobile B200 kernels: status plumbing, the
// real spherical-harmonic polynomials (e3nn "component" normalisation) and
// small launch utilities.  Everything here is internal to libbatmobile_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "batmobile_b200.h"
#include "cg_l3.h"

namespace bm {

constexpr int kIrreps = 16;     // (L_max + 1)^2 for L_max = 3
constexpr int kNumSMs = 148;    // B200

// Records a human-readable message for bm_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Maps a CUDA error (from the launch just made) to a bm status and adds
// `launches` to the process-wide kernel launch counter (bm_launch_count).
int check_launch(const char* what, int launches = 1);
// The CUDA context current on this thread (driver handle, nullptr if none).
// Per-device caches of symbol addresses are keyed by it, so that a device
// reset or a new primary context makes them resolve the address again.
void* current_context();

// Runtime-indexable copies of the per-group tables of cg_l3.h (device code
// cannot index host constexpr arrays with a runtime value).
constexpr int kSO0 = kGroupSlotOff[0], kSO1 = kGroupSlotOff[1], kSO2 = kGroupSlotOff[2],
              kSO3 = kGroupSlotOff[3], kSO4 = kGroupSlotOff[4];
constexpr int kGP0 = kGroupPaths[0], kGP1 = kGroupPaths[1], kGP2 = kGroupPaths[2], kGP3 = kGroupPaths[3];
__host__ __device__ __forceinline__ int group_slot_off(int g) {
  return g <= 0 ? kSO0 : g == 1 ? kSO1 : g == 2 ? kSO2 : g == 3 ? kSO3 : kSO4;
}
__host__ __device__ __forceinline__ int group_paths(int g) {
  return g <= 0 ? kGP0 : g == 1 ? kGP1 : g == 2 ? kGP2 : kGP3;
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Packed fp32 pair FMA (sm_100 f32x2): d = a * b + d lane-wise, one instruction.
__device__ __forceinline__ void ffma2(float2& d, float2 a, float2 b) {
  unsigned long long dd = (unsigned long long)__float_as_uint(d.x) | ((unsigned long long)__float_as_uint(d.y) << 32);
  const unsigned long long aa =
      (unsigned long long)__float_as_uint(a.x) | ((unsigned long long)__float_as_uint(a.y) << 32);
  const unsigned long long bb =
      (unsigned long long)__float_as_uint(b.x) | ((unsigned long long)__float_as_uint(b.y) << 32);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(dd) : "l"(aa), "l"(bb));
  d.x = __uint_as_float((unsigned)dd);
  d.y = __uint_as_float((unsigned)(dd >> 32));
}

// Warp-level tf32 tensor-core MMA (mma.sync m16n8k8, fp32 accumulate) and the
// hi/lo split of an fp32 operand for the 3-pass product hi*hi + hi*lo + lo*hi
// (about fp32 accuracy).  Fragment layout (g = lane / 4, t = lane % 4):
// A: a0 = A[g][t], a1 = A[g+8][t], a2 = A[g][t+4], a3 = A[g+8][t+4];
// B: b0 = B[t][g], b1 = B[t+4][g];  D: d0 = D[g][2t], d1 = D[g][2t+1],
// d2 = D[g+8][2t], d3 = D[g+8][2t+1].
__device__ __forceinline__ void mma_tf32_16x8x8(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// v = hi + lo with hi = v truncated to tf32 (sign, exponent and the top 10
// mantissa bits: one logic op on the integer pipe rather than a conversion) and
// lo = v - hi exactly; the MMA reads the top bits of lo, so hi*hi + hi*lo + lo*hi
// misses about 2^-20 |a b| (the lo*lo term and lo's own truncation)
__device__ __forceinline__ void split_tf32(float v, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(v) & 0xFFFFE000u;
  lo = __float_as_uint(v - __uint_as_float(hi));
}

inline unsigned grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  return (unsigned)(g > 0 ? g : 1);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#define BM_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) return ::bm::set_error(BM_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

// ---------------------------------------------------------------------------
// Real spherical harmonics, component normalisation (|Y_l|^2 = 2l+1 on the
// unit sphere), polynomial form.  Component order inside each l follows the
// reference kernel src/spherical_harmonics/spherical_harmonics.cu:56-96
// (l=1 is sqrt(3)*(x, y, z)); l=4..6 use e3nn's recurrence on l-1 times
// (x, y, z) as in spherical_harmonics.cu:99-256.
// ---------------------------------------------------------------------------
// Forward-mode dual number (value and d/dx, d/dy, d/dz): evaluating the SH
// polynomials / recurrence on duals gives their exact Jacobian.
struct D3 {
  float v, dx, dy, dz;
  __device__ __forceinline__ D3() {}
  __device__ __forceinline__ D3(float c) : v(c), dx(0.0f), dy(0.0f), dz(0.0f) {}
  __device__ __forceinline__ D3(float a, float b, float c, float d) : v(a), dx(b), dy(c), dz(d) {}
};
__device__ __forceinline__ D3 operator+(D3 a, D3 b) { return D3(a.v + b.v, a.dx + b.dx, a.dy + b.dy, a.dz + b.dz); }
__device__ __forceinline__ D3 operator-(D3 a, D3 b) { return D3(a.v - b.v, a.dx - b.dx, a.dy - b.dy, a.dz - b.dz); }
__device__ __forceinline__ D3 operator-(D3 a) { return D3(-a.v, -a.dx, -a.dy, -a.dz); }
__device__ __forceinline__ D3 operator*(D3 a, D3 b) {
  return D3(a.v * b.v, a.dx * b.v + a.v * b.dx, a.dy * b.v + a.v * b.dy, a.dz * b.v + a.v * b.dz);
}
__device__ __forceinline__ D3 operator*(float c, D3 a) { return D3(c * a.v, c * a.dx, c * a.dy, c * a.dz); }
__device__ __forceinline__ D3 operator*(D3 a, float c) { return c * a; }

template <int L, class T = float>
__device__ __forceinline__ void sh_eval(T x, T y, T z, T* o) {
  o[0] = 1.0f;
  if (L < 1) return;
  const float s3 = 1.7320508075688772f;
  o[1] = s3 * x; o[2] = s3 * y; o[3] = s3 * z;
  if (L < 2) return;
  const float s15 = 3.872983346207417f, s5 = 2.23606797749979f;
  const T xx = x * x, yy = y * y, zz = z * z, xz2 = xx + zz;
  const T q0 = s15 * x * z;            // l=2, m=-2
  const T q4 = 0.5f * s15 * (zz - xx); // l=2, m=+2
  o[4] = q0;
  o[5] = s15 * x * y;
  o[6] = s5 * (yy - 0.5f * xz2);
  o[7] = s15 * y * z;
  o[8] = q4;
  if (L < 3) return;
  const float k0 = 1.0801234497346432f, k1 = 2.6457513110645907f;
  const float k2 = 1.6201851746019651f, k3 = 1.3228756555322954f;
  const T t = 4.0f * yy - xz2;
  o[9] = k0 * (q0 * z + q4 * x);
  o[10] = k1 * q0 * y;
  o[11] = k2 * t * x;
  o[12] = k3 * y * (2.0f * yy - 3.0f * xz2);
  o[13] = k2 * z * t;
  o[14] = k1 * q4 * y;
  o[15] = k0 * (q4 * z - q0 * x);
  if (L < 4) return;
  {
    const T* a = o + 9;
    T* b = o + 16;
    b[0] = 1.0606601717798214f * (a[0] * z + a[6] * x);
    b[1] = 0.75f * a[0] * y + 0.9185586535436917f * a[1] * z + 0.9185586535436917f * a[5] * x;
    b[2] = -0.2004459314343183f * a[0] * z + 0.9819805060619656f * a[1] * y +
           0.7763237542601484f * a[2] * z + 0.7763237542601484f * a[4] * x +
           0.2004459314343183f * a[6] * x;
    b[3] = -0.3471825374147068f * a[1] * z + 1.0978875820670997f * a[2] * y +
           0.8964214570007952f * a[3] * x + 0.3471825374147068f * a[5] * x;
    b[4] = -0.6943650748294136f * a[2] * x + 1.1338934190276817f * a[3] * y -
           0.6943650748294136f * a[4] * z;
    b[5] = -0.3471825374147068f * a[1] * x + 0.8964214570007952f * a[3] * z +
           1.0978875820670997f * a[4] * y - 0.3471825374147068f * a[5] * z;
    b[6] = -0.2004459314343183f * a[0] * x - 0.7763237542601484f * a[2] * x +
           0.7763237542601484f * a[4] * z + 0.9819805060619656f * a[5] * y -
           0.2004459314343183f * a[6] * z;
    b[7] = -0.9185586535436917f * a[1] * x + 0.9185586535436917f * a[5] * z + 0.75f * a[6] * y;
    b[8] = 1.0606601717798214f * (-a[0] * x + a[6] * z);
  }
  if (L < 5) return;
  {
    const T* a = o + 16;
    T* b = o + 25;
    b[0] = 1.0488088481701516f * (a[0] * z + a[8] * x);
    b[1] = 0.6633249580710801f * a[0] * y + 0.9380831519646859f * a[1] * z + 0.9380831519646859f * a[7] * x;
    b[2] = -0.1563471919941143f * a[0] * z + 0.8844332774281066f * a[1] * y +
           0.8273115763993905f * a[2] * z + 0.8273115763993905f * a[6] * x +
           0.1563471919941143f * a[8] * x;
    b[3] = -0.2708012801545320f * a[1] * z + 1.0132456102380443f * a[2] * y +
           0.7164728420068226f * a[3] * z + 0.7164728420068226f * a[5] * x +
           0.2708012801545320f * a[7] * x;
    b[4] = -0.3829708431025353f * a[2] * z + 1.0832051206181281f * a[3] * y +
           0.8563488385776753f * a[4] * x + 0.3829708431025353f * a[6] * x;
    b[5] = -0.6992058987801010f * a[3] * x + 1.1055415967851332f * a[4] * y - 0.6992058987801010f * a[5] * z;
    b[6] = -0.3829708431025353f * a[2] * x + 0.8563488385776753f * a[4] * z +
           1.0832051206181281f * a[5] * y - 0.3829708431025353f * a[6] * z;
    b[7] = -0.2708012801545320f * a[1] * x - 0.7164728420068226f * a[3] * x +
           0.7164728420068226f * a[5] * z + 1.0132456102380443f * a[6] * y -
           0.2708012801545320f * a[7] * z;
    b[8] = -0.1563471919941143f * a[0] * x - 0.8273115763993905f * a[2] * x +
           0.8273115763993905f * a[6] * z + 0.8844332774281066f * a[7] * y -
           0.1563471919941143f * a[8] * z;
    b[9] = -0.9380831519646859f * a[1] * x + 0.9380831519646859f * a[7] * z + 0.6633249580710801f * a[8] * y;
    b[10] = 1.0488088481701516f * (-a[0] * x + a[8] * z);
  }
  if (L < 6) return;
  {
    const T* a = o + 25;
    T* b = o + 36;
    b[0] = 1.0408329997330663f * (a[0] * z + a[10] * x);
    b[1] = 0.6009252125773314f * a[0] * y + 0.9501461875826149f * a[1] * z + 0.9501461875826149f * a[9] * x;
    b[2] = -0.1281176857976346f * a[0] * z + 0.8102873913406630f * a[1] * y +
           0.1281176857976346f * a[10] * x + 0.8594395636904107f * a[2] * z +
           0.8594395636904107f * a[8] * x;
    b[3] = -0.2219063411496486f * a[1] * z + 0.9414688716912718f * a[2] * y +
           0.7687061147858074f * a[3] * z + 0.7687061147858074f * a[7] * x +
           0.2219063411496486f * a[9] * x;
    b[4] = -0.3138229572304240f * a[2] * z + 1.0249414863810766f * a[3] * y +
           0.6779350703393059f * a[4] * z + 0.6779350703393059f * a[6] * x +
           0.3138229572304240f * a[8] * x;
    b[5] = -0.4051436956703315f * a[3] * z + 1.0719094639893330f * a[4] * y +
           0.8302975005345611f * a[5] * x + 0.4051436956703315f * a[7] * x;
    b[6] = -0.7017294652672371f * a[4] * x + 1.0871146130092180f * a[5] * y - 0.7017294652672371f * a[6] * z;
    b[7] = -0.4051436956703315f * a[3] * x + 0.8302975005345611f * a[5] * z +
           1.0719094639893330f * a[6] * y - 0.4051436956703315f * a[7] * z;
    b[8] = -0.3138229572304240f * a[2] * x - 0.6779350703393059f * a[4] * x +
           0.6779350703393059f * a[6] * z + 1.0249414863810766f * a[7] * y -
           0.3138229572304240f * a[8] * z;
    b[9] = -0.2219063411496486f * a[1] * x - 0.7687061147858074f * a[3] * x +
           0.7687061147858074f * a[7] * z + 0.9414688716912718f * a[8] * y -
           0.2219063411496486f * a[9] * z;
    b[10] = -0.1281176857976346f * a[0] * x - 0.1281176857976346f * a[10] * z -
            0.8594395636904107f * a[2] * x + 0.8594395636904107f * a[8] * z +
            0.8102873913406630f * a[9] * y;
    b[11] = -0.9501461875826149f * a[1] * x + 0.6009252125773314f * a[10] * y + 0.9501461875826149f * a[9] * z;
    b[12] = 1.0408329997330663f * (-a[0] * x + a[10] * z);
  }
}

// Gradient of sum_lm g[lm] * Y_lm(x, y, z) with respect to (x, y, z) for
// L_max <= 3; the raw polynomial Jacobian, not projected onto the sphere
// (reference: src/spherical_harmonics/spherical_harmonics_backward.cu:25-200,
// python/batmobile/autograd.py:97-281).
template <int L>
__device__ __forceinline__ void sh_grad(float x, float y, float z, const float* g,
                                        float& gx, float& gy, float& gz) {
  gx = gy = gz = 0.0f;
  if (L < 1) return;
  const float s3 = 1.7320508075688772f;
  gx += s3 * g[1]; gy += s3 * g[2]; gz += s3 * g[3];
  if (L < 2) return;
  const float s15 = 3.872983346207417f, s5 = 2.23606797749979f;
  gx += s15 * (z * g[4] + y * g[5]) - s5 * x * g[6] - s15 * x * g[8];
  gy += s15 * (x * g[5] + z * g[7]) + 2.0f * s5 * y * g[6];
  gz += s15 * (x * g[4] + y * g[7]) - s5 * z * g[6] + s15 * z * g[8];
  if (L < 3) return;
  const float k0 = 1.0801234497346432f * s15, k1 = 2.6457513110645907f * s15;
  const float k2 = 1.6201851746019651f, k3 = 1.3228756555322954f;
  const float xx = x * x, yy = y * y, zz = z * z;
  // Y9  = k0 (1.5 x z^2 - 0.5 x^3)       Y15 = k0 (0.5 z^3 - 1.5 x^2 z)
  // Y10 = k1 x y z                        Y14 = 0.5 k1 (z^2 - x^2) y
  // Y11 = k2 (4y^2 - x^2 - z^2) x         Y13 = k2 (4y^2 - x^2 - z^2) z
  // Y12 = k3 y (2y^2 - 3x^2 - 3z^2)
  const float g9 = g[9], g10 = g[10], g11 = g[11], g12 = g[12], g13 = g[13], g14 = g[14], g15 = g[15];
  gx += k0 * 1.5f * (zz - xx) * g9 + k1 * y * z * g10 + k2 * (4.0f * yy - 3.0f * xx - zz) * g11 -
        6.0f * k3 * x * y * g12 - 2.0f * k2 * x * z * g13 - k1 * x * y * g14 - 3.0f * k0 * x * z * g15;
  gy += k1 * x * z * g10 + 8.0f * k2 * x * y * g11 + k3 * (6.0f * yy - 3.0f * (xx + zz)) * g12 +
        8.0f * k2 * y * z * g13 + 0.5f * k1 * (zz - xx) * g14;
  gz += 3.0f * k0 * x * z * g9 + k1 * x * y * g10 - 2.0f * k2 * x * z * g11 - 6.0f * k3 * y * z * g12 +
        k2 * (4.0f * yy - xx - 3.0f * zz) * g13 + k1 * y * z * g14 + k0 * 1.5f * (zz - xx) * g15;
}

// Unit vector with the clamp of the reference interaction block
// (benchmarks/benchmark_e2e_mace.py:328-329: norm.clamp(min=1e-8)).
constexpr float kNormEps = 1e-8f;
__device__ __forceinline__ float unit3(float& x, float& y, float& z) {
  float r = sqrtf(x * x + y * y + z * z);
  float d = fmaxf(r, kNormEps);
  x = x / d; y = y / d; z = z / d;
  return r;
}

// Chain rule through v -> v / max(|v|, eps): given d/d(unit), the gradient
// w.r.t. v.  Above eps it is (g - u (u.g)) / |v|; clamped vectors scale by 1/eps
// (the clamp has zero derivative), matching torch autograd on the reference code.
__device__ __forceinline__ void unit3_backward(float ux, float uy, float uz, float r,
                                               float& gx, float& gy, float& gz) {
  if (r >= kNormEps) {
    float d = ux * gx + uy * gy + uz * gz;
    gx = (gx - ux * d) / r; gy = (gy - uy * d) / r; gz = (gz - uz * d) / r;
  } else {
    gx /= kNormEps; gy /= kNormEps; gz /= kNormEps;
  }
}

// Exclusive scan of int32 counts into int64 offsets (n+1 outputs, out[n] = total).
// Deterministic three-phase scan; `tmp` must hold scan_tmp_elems(n) int64.
size_t scan_tmp_elems(int64_t n);
int exclusive_scan_i32_to_i64(const int* in, int64_t* out, int64_t n, int64_t* tmp, cudaStream_t st);

// Sort the values of every CSR row ascending (rows are short: used for
// deterministic edge order).  vals may be int32 or int64.
int sort_rows_i64(const int64_t* row_ptr, int64_t* vals, int64_t n_rows, cudaStream_t st);

}  // namespace bm
