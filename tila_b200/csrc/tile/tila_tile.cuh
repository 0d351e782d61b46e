// tila_tile.cuh - sm_100a tile-primitive library used by the kernels that the
// B200 backend generates from Tila's typed TIR.  Header-only; compiled by
// NVRTC together with each generated kernel (no host headers are needed).
//
// Contents
//   * scalar semantics of Tila's dtypes (f16/bf16 rounding through f32 the way
//     NumPy computes them, wrapping integer arithmetic, floor division,
//     NaN-propagating max) - interp.py:199-333 / numeric.py:56-78 / ADR-008;
//   * warp/CTA reduction building blocks;
//   * mbarrier helpers whose waits are bounded and report a timeout through
//     the kernel's error word instead of hanging;
//   * TMA tile loads (cp.async.bulk.tensor, no multicast);
//   * tcgen05 tensor-memory allocation, MMA (kind::f16, f32 accumulate),
//     commit, tcgen05.ld/st, and shared-memory matrix descriptors.
#pragma once

namespace tila {

typedef signed char i8;
typedef short i16;
typedef int i32;
typedef long long i64;
typedef unsigned char u8;
typedef unsigned short u16;
typedef unsigned int u32;
typedef unsigned long long u64;

// ---------------------------------------------------------------------------
// error reporting
// ---------------------------------------------------------------------------

enum ErrorCode : u32 {
  kErrNone = 0,
  kErrMbarrierTimeout = 1,   // a bounded mbarrier wait gave up
  kErrTmemAlloc = 2,         // tensor memory allocation failed
  kErrAssumption = 3,        // a ti.assume predicate was false (debug builds)
  kErrSchedule = 4,          // a warp-specialised loop chain was not contiguous at run time
};

// Records the first error of a launch.  `err` points at the launch's 16-byte
// error block: word 0 takes (code << 24) | line of the first error; bytes
// 8-15 hold the device address of a notification word in page-locked host
// memory (0 = none), where the thread that recorded the error also stores it,
// so that the host sees device errors without synchronising.
__device__ __forceinline__ void report_error(u32 *err, u32 code, u32 where) {
  if (err == nullptr) return;
  const u32 v = (code << 24) | (where & 0xFFFFFFu);
  if (atomicCAS(err, 0u, v) == 0u) {
    const u64 notify = *reinterpret_cast<volatile u64 *>(err + 2);
    if (notify != 0) {
      *reinterpret_cast<volatile u32 *>(notify) = v;
      __threadfence_system();
    }
  }
}

// ---------------------------------------------------------------------------
// dtype semantics
// ---------------------------------------------------------------------------

// f16 <-> f32 with NumPy's NaN handling (npy_halfbits_to_floatbits and
// npy_floatbits_to_halfbits): a NaN keeps its sign and the top bits of its
// payload, so a half value that only moves through f32 (a copy, a reshape)
// comes back bit for bit.
__device__ __forceinline__ float h2f(u16 h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  if ((h & 0x7FFFu) > 0x7C00u)
    f = __uint_as_float((static_cast<u32>(h & 0x8000u) << 16) | 0x7F800000u |
                        (static_cast<u32>(h & 0x3FFu) << 13));
  return f;
}
__device__ __forceinline__ u16 f2h(float f) {
  u16 h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  const u32 b = __float_as_uint(f);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) {
    u32 r = 0x7C00u + ((b & 0x7FFFFFu) >> 13);
    if (r == 0x7C00u) r += 1u;               // a payload below the kept bits stays a NaN
    h = static_cast<u16>(((b >> 16) & 0x8000u) | r);
  }
  return h;
}
__device__ __forceinline__ u16 d2h(double d) {
  u16 h;
  asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(d));
  return h;
}
__device__ __forceinline__ float bf2f(u16 h) {
  return __uint_as_float(static_cast<u32>(h) << 16);
}
// f32 -> bf16, round to nearest even; a NaN keeps its sign and the top bits of
// its payload (a bf16 value that only moves through f32 comes back bit for bit).
__device__ __forceinline__ u16 f2bf(float f) {
  u16 h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
  const u32 b = __float_as_uint(f);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) {
    u32 r = b >> 16;
    if ((r & 0x7Fu) == 0u) r |= 0x40u;      // a payload below the kept bits stays a NaN
    h = static_cast<u16>(r);
  }
  return h;
}
__device__ __forceinline__ u16 d2bf(double d) {
  // f64 -> bf16 with a single rounding: round to f32 with round-to-odd first
  // so that the second rounding cannot create a double-rounding error.
  float f;
  asm("cvt.rn.f32.f64 %0, %1;" : "=f"(f) : "d"(d));
  double back = static_cast<double>(f);
  if (back != d && !(d != d)) {
    u32 bits = __float_as_uint(f);
    if ((bits & 1u) == 0u) {
      // move one ulp towards d to make the f32 intermediate odd
      bits = (back < d) == (f >= 0.0f) ? bits + 1u : bits - 1u;
      f = __uint_as_float(bits);
    }
  }
  return f2bf(f);
}
// Two f32 -> one f16x2 word (lo in bits 0..15), each rounded to nearest even.
__device__ __forceinline__ u32 pack_f16x2(float lo, float hi) {
  u32 r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 2^x with the hardware approximation: maximum relative error 2^-22.5,
// subnormal results supported, exp2(-inf) = +0, exp2(+inf) = +inf, NaN -> NaN.
__device__ __forceinline__ float exp2_fast(float x) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// 2^x for arguments >= -126 (normal results): the flush-to-zero form, equal
// to exp2_fast there.
__device__ __forceinline__ float exp2_ftz(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Division by a divisor shared by many dividends (a row sum broadcast along
// a row, a scalar parameter): the IEEE f32 quotient a / b, bit for bit, with
// the reciprocal computed once per divisor.
// Method: residual correction after P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990 (Markstein's theorem: if q is a faithful approximation of a/b and y
// approximates 1/b with relative error below 2^-24, then r = a - b*q is exact
// and RN(q + r*y) = RN(a/b), barring underflow and overflow).  q0 = RN(a*y)
// with y = RN(1/b) can be off by up to 1.5 ulp (e.g. 1.5 / 1.9999999), so a
// first correction makes it faithful (its error is then below 0.5 ulp plus
// 2^-45 relative) and the second one rounds correctly.  Magnitudes in
// [2^-60, 2^60) for both operands (and zero for the dividend) keep every
// intermediate normal and finite.  A thread first records its dividends'
// range (udiv_track); if one leaves it (subnormals, infinities, NaN, extreme
// exponents) the thread divides with IEEE division instead (udiv_all_fast).
// Tracking before dividing lets the quotients overwrite the dividends'
// registers.
struct UDiv {
  float b;      // the divisor
  float y;      // RN(1/b)
  bool ok;      // 2^-60 <= |b| < 2^60
};
__device__ __forceinline__ UDiv udiv_prepare(float b) {
  UDiv d;
  const u32 ub = __float_as_uint(b);
  d.b = b;
  d.y = __frcp_rn(b);
  d.ok = ((ub & 0x7fffffffu) - 0x21800000u) < (0x5d800000u - 0x21800000u);
  return d;
}
// Range record of one dividend: hi = max of |a| (NaN propagates), lo = min
// of (2|a| bits) - 1 (a zero dividend maps to 0xffffffff and so leaves it).
__device__ __forceinline__ void udiv_track(float a, float &hi, u32 &lo) {
  const u32 ua = __float_as_uint(a);
  asm("max.NaN.f32 %0, %0, %1;" : "+f"(hi) : "f"(fabsf(a)));
  lo = min(lo, ua + ua - 1u);
}
// Quotient of a recorded dividend (valid when udiv_all_fast holds).  The
// first product p = a*y carries the sign of a/b, also for a zero dividend;
// the corrections can turn a -0 quotient into +0 but never the reverse, so
// OR-ing p's sign bit restores it (and changes nothing for other quotients).
__device__ __forceinline__ float udiv_q(float a, const UDiv &d) {
  const float p = __fmul_rn(a, d.y);
  float r = __fmaf_rn(-d.b, p, a);
  float q = __fmaf_rn(r, d.y, p);
  r = __fmaf_rn(-d.b, q, a);
  q = __fmaf_rn(r, d.y, q);
  return __uint_as_float(__float_as_uint(q) | (__float_as_uint(p) & 0x80000000u));
}
__device__ __forceinline__ bool udiv_all_fast(const UDiv &d, float hi, u32 lo) {
  return d.ok && hi < 0x1p60f && lo >= 0x42ffffffu;   // |a| in [2^-60, 2^60) or zero
}

// Packed f32 pairs (sm_100 f32x2 arithmetic): each lane is rounded exactly
// like the scalar operation, two elements per instruction.
__device__ __forceinline__ u64 pk2(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float lo2(u64 v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return a;
}
__device__ __forceinline__ float hi2(u64 v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return b;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Two quotients by the same divisor with f32x2 arithmetic (same steps and
// results as two udiv_q calls).
__device__ __forceinline__ void udiv_q2(float a0, float a1, const UDiv &d, float &q0, float &q1) {
  const u64 a = pk2(a0, a1), y = pk2(d.y, d.y), nb = pk2(-d.b, -d.b);
  const u64 p = mul2(a, y);
  u64 r = fma2(nb, p, a);
  u64 q = fma2(r, y, p);
  r = fma2(nb, q, a);
  q = fma2(r, y, q);
  q0 = __uint_as_float(__float_as_uint(lo2(q)) | (__float_as_uint(lo2(p)) & 0x80000000u));
  q1 = __uint_as_float(__float_as_uint(hi2(q)) | (__float_as_uint(hi2(p)) & 0x80000000u));
}

// Round an f32 to the nearest f16 / bf16 value and widen back (the register
// representation of f16/bf16 tiles is an f32 holding a representable value).
__device__ __forceinline__ float round_f16(float f) { return h2f(f2h(f)); }
__device__ __forceinline__ float round_bf16(float f) { return bf2f(f2bf(f)); }

// NumPy's maximum propagates NaN (ADR-008); PTX max.NaN does the same.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ double max_nan(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  return a > b ? a : b;
}
template <typename T>
__device__ __forceinline__ T max_int(T a, T b) { return a > b ? a : b; }

// Wrapping integer arithmetic: compute in the unsigned type of the same width.
template <typename T> struct Unsigned;
template <> struct Unsigned<i8> { typedef u8 type; };
template <> struct Unsigned<i16> { typedef u16 type; };
template <> struct Unsigned<i32> { typedef u32 type; };
template <> struct Unsigned<i64> { typedef u64 type; };
template <> struct Unsigned<u8> { typedef u8 type; };
template <> struct Unsigned<u16> { typedef u16 type; };
template <> struct Unsigned<u32> { typedef u32 type; };
template <> struct Unsigned<u64> { typedef u64 type; };

template <typename T>
__device__ __forceinline__ T wadd(T a, T b) {
  typedef typename Unsigned<T>::type U;
  return static_cast<T>(static_cast<U>(static_cast<U>(a) + static_cast<U>(b)));
}
template <typename T>
__device__ __forceinline__ T wsub(T a, T b) {
  typedef typename Unsigned<T>::type U;
  return static_cast<T>(static_cast<U>(static_cast<U>(a) - static_cast<U>(b)));
}
template <typename T>
__device__ __forceinline__ T wmul(T a, T b) {
  typedef typename Unsigned<T>::type U;
  return static_cast<T>(static_cast<U>(static_cast<U>(a) * static_cast<U>(b)));
}
template <typename T>
__device__ __forceinline__ T wneg(T a) {
  typedef typename Unsigned<T>::type U;
  return static_cast<T>(static_cast<U>(U(0) - static_cast<U>(a)));
}

// Floor division and modulo with Python semantics; MIN // -1 wraps to MIN
// and MIN % -1 is 0 (lowering.py:24-38).  Division by zero is excluded by
// the launch-time integer gate.
template <typename T>
__device__ __forceinline__ T floordiv(T a, T b, T minv) {
  if (static_cast<T>(-1) > static_cast<T>(0)) return b == 0 ? T(0) : a / b;  // unsigned
  if (a == minv && b == static_cast<T>(-1)) return minv;
  if (b == 0) return T(0);
  T q = a / b;
  T r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) q = q - 1;
  return q;
}
template <typename T>
__device__ __forceinline__ T floormod(T a, T b, T minv) {
  if (static_cast<T>(-1) > static_cast<T>(0)) return b == 0 ? T(0) : a % b;
  if (a == minv && b == static_cast<T>(-1)) return T(0);
  if (b == 0) return T(0);
  T r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) r = r + b;
  return r;
}

// Python float floor division / modulo (NumPy's npy_divmod): the remainder
// takes the divisor's sign and the quotient is floor((a - mod) / b).
template <typename F>
__device__ __forceinline__ F py_mod(F a, F b) {
  F m = fmod(a, b);
  if (m != F(0)) {
    if ((b < F(0)) != (m < F(0))) m += b;
  } else {
    m = copysign(F(0), b);
  }
  return m;
}
template <typename F>
__device__ __forceinline__ F py_floordiv(F a, F b) {
  if (b == F(0)) return a / b;
  F m = fmod(a, b);
  F div = (a - m) / b;
  if (m != F(0) && ((b < F(0)) != (m < F(0)))) div -= F(1);
  F fl;
  if (div != F(0)) {
    fl = floor(div);
    if (div - fl > F(0.5)) fl += F(1);
  } else {
    fl = copysign(F(0), a / b);
  }
  return fl;
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------

struct SumOp {
  template <typename T> __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
};
struct MaxOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return max_nan(a, b); }
  __device__ __forceinline__ double operator()(double a, double b) const { return max_nan(a, b); }
  template <typename T> __device__ __forceinline__ T operator()(T a, T b) const { return max_int(a, b); }
};
struct WrapSumOp {
  template <typename T> __device__ __forceinline__ T operator()(T a, T b) const { return wadd(a, b); }
};

template <typename T>
__device__ __forceinline__ T shfl_xor(T v, int mask) {
  return __shfl_xor_sync(0xffffffffu, v, mask);
}
__device__ __forceinline__ double shfl_xor(double v, int mask) {
  return __shfl_xor_sync(0xffffffffu, v, mask);
}
__device__ __forceinline__ bool shfl_xor(bool v, int mask) {
  return __shfl_xor_sync(0xffffffffu, static_cast<int>(v), mask) != 0;
}

// ---------------------------------------------------------------------------
// shared memory / proxies
// ---------------------------------------------------------------------------

__device__ __forceinline__ u32 smem_u32(const void *p) {
  return static_cast<u32>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier (bounded waits)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(u64 *bar, u32 count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(u64 *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(u64 *bar, u32 bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(u64 *bar, u32 parity) {
  u32 ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Programmatic dependent launch.  A kernel launched with the overlap flag may
// be resident before the previous grid in its stream has finished;
// grid_dep_wait blocks until that grid has completed and its memory writes are
// visible, and must precede every global-memory access.  grid_dep_release
// lets the next grid in the stream be scheduled once every CTA of this grid
// has executed it (it does not make this grid's results visible early: the
// dependent's own wait still covers them).  Without the flag both are no-ops.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Hint: bring the 128-byte line holding `p` into L2.  Issued before
// grid_dep_wait for a program's first loads, so their DRAM traffic overlaps
// the previous grid; L2 is the point of coherence, so the loads after the
// wait still observe everything the previous grid wrote.
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ void grid_dep_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Barrier over the whole CTA (both warpgroups in two-program mode).
__device__ __forceinline__ void cta_sync() { __syncthreads(); }
// Barrier of one 128-thread warpgroup (named barrier 1 + wg) in kernels that
// run one program per warpgroup.
__device__ __forceinline__ void wg_sync(int wg) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
}

// Barrier of the `n` threads of program `wg` (named barrier 1 + wg) in kernels
// that run one program per group of n threads.
__device__ __forceinline__ void wg_sync_n(int wg, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "r"(n) : "memory");
}

__device__ __forceinline__ u64 globaltimer_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Time limit of one mbarrier wait.  A healthy wait ends in microseconds; a
// wait that reaches this limit is treated as dead.
#ifndef TILA_WAIT_NS
#define TILA_WAIT_NS 1000000000ull
#endif

// Waits for the phase with the given parity to complete.  Returns false (and
// records kErrMbarrierTimeout) when the time limit passes; callers stop
// issuing work and fall through to their cleanup.  `*dead` is shared state:
// once any wait failed, later waits return immediately.
__device__ __forceinline__ bool mbar_wait(u64 *bar, u32 parity, u32 *err, u32 where,
                                          volatile int *dead) {
  if (mbar_try_wait(bar, parity)) return true;
  const u64 start = globaltimer_ns();
  for (u32 i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (dead != nullptr && *dead) return false;
      if (globaltimer_ns() - start > TILA_WAIT_NS) break;
    }
  }
  report_error(err, kErrMbarrierTimeout, where);
  if (dead != nullptr) *dead = 1;
  return false;
}

// Hand-off flags between CTAs of one grid (global memory, GPU scope): a CTA
// writes data, synchronises its threads, and one thread releases the flag; a
// reader acquires it (bounded wait) and synchronises its threads before
// reading the data.
__device__ __forceinline__ void flag_release(u32 *flag, u32 v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}
__device__ __forceinline__ u32 flag_acquire(const u32 *flag) {
  u32 v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  return v;
}
// Wait until *flag == v; on timeout record kErrMbarrierTimeout, mark the CTA
// dead and return false (the writer is a CTA of the same grid that runs at
// the same time or earlier, so the wait ends unless something failed).
__device__ __forceinline__ bool flag_wait(const u32 *flag, u32 v, u32 *err, u32 where,
                                          volatile int *dead) {
  if (flag_acquire(flag) == v) return true;
  const u64 start = globaltimer_ns();
  for (u32 i = 1;; ++i) {
    if (flag_acquire(flag) == v) return true;
    if ((i & 63u) == 0u) {
      if (dead != nullptr && *dead) return false;
      if (globaltimer_ns() - start > TILA_WAIT_NS) break;
    }
  }
  report_error(err, kErrMbarrierTimeout, where);
  if (dead != nullptr) *dead = 1;
  return false;
}

// ---------------------------------------------------------------------------
// TMA (tensor memory accelerator) tile loads - single CTA, no multicast
// ---------------------------------------------------------------------------

struct __align__(64) TensorMap { u64 opaque[16]; };

__device__ __forceinline__ void tma_prefetch_desc(const TensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const TensorMap *map, u64 *bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<u64>(map)), "r"(smem_u32(bar)),
        "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const TensorMap *map, u64 *bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<u64>(map)), "r"(smem_u32(bar)),
        "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const TensorMap *map, u64 *bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<u64>(map)), "r"(smem_u32(bar)),
        "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// TMA tile stores (shared -> global).  Elements of the box outside the
// tensor are not written.  The issuing thread groups its stores with
// bulk_commit() and must call bulk_wait_read() before the shared-memory
// source is overwritten or the CTA exits.  Coordinates must be >= 0.
__device__ __forceinline__ void tma_store_2d(const TensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<u64>(map)), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_store_3d(const TensorMap *map, const void *src, int x, int y,
                                             int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<u64>(map)), "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const TensorMap *map, const void *src, int x, int y,
                                             int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
               ::"l"(reinterpret_cast<u64>(map)), "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z),
                 "r"(w) : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read_n() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation tensor core
// ---------------------------------------------------------------------------

// Per-warpgroup register budgets (setmaxnreg): executed by every thread of a
// warpgroup.  reg_dealloc returns registers to the CTA's pool; reg_alloc waits
// until the pool (threads at launch x registers per thread at launch) holds
// enough free registers, so the budgets of all warpgroups must add up to at
// most that total.
template <u32 N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <u32 N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Allocates `ncols` (power of two >= 32) TMEM columns; executed by one whole
// warp.  The base address is written to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(u32 *slot, u32 ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(slot)), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(u32 taddr, u32 ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset, [52] LBO mode, [61,64) swizzle mode
//   (0 none, 2 = 128B, 4 = 64B, 6 = 32B).
// Built from a precomputed base: base4 = (shared address of the dynamic
// shared memory) >> 4 and a 16-byte aligned offset; the LBO / SBO / swizzle
// fields are compile-time constants, so a descriptor costs one add and one OR
// (the MMA-issuing thread would otherwise spend more time building
// descriptors than an N <= 128 instruction takes to execute).  Shared
// addresses stay below 2^18, so the start-address field cannot carry into LBO.
template <u32 LBO, u32 SBO, u32 SW>
__device__ __forceinline__ u64 sdesc(u32 base4, u32 off) {
  constexpr u64 fields = (static_cast<u64>((LBO >> 4) & 0x3FFFu) << 16) |
                         (static_cast<u64>((SBO >> 4) & 0x3FFFu) << 32) |
                         (static_cast<u64>(1) << 46) | (static_cast<u64>(SW & 7u) << 61);
  return fields | static_cast<u64>(base4 + (off >> 4));
}

// Instruction descriptor for kind::f16 with f16 inputs and f32 accumulate:
//   [4,6) D format (1 = f32), [7,10) A format (0 = f16), [10,13) B format,
//   [15] A major (0 = K-major, 1 = MN-major), [16] B major,
//   [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr u32 idesc_f16_f32(u32 m, u32 n, u32 a_mn_major, u32 b_mn_major) {
  return (1u << 4) | (a_mn_major << 15) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]; issued by a single thread.
__device__ __forceinline__ void mma_f16_ss(u32 d_tmem, u64 a_desc, u64 b_desc, u32 idesc,
                                           u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]; A is read from tensor memory.
__device__ __forceinline__ void mma_f16_ts(u32 d_tmem, u32 a_tmem, u64 b_desc, u32 idesc,
                                           u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread are done.
__device__ __forceinline__ void mma_commit(u64 *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// tcgen05.ld / st, shape 32x32b: lane i of the warp accesses TMEM lane
// (32 * (warp % 4) + i), registers walk consecutive columns.
__device__ __forceinline__ void tmem_ld8(u32 taddr, float *v) {
  u32 r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld32(u32 taddr, float *v) {
  u32 r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st8(u32 taddr, const float *v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
                 "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
                 "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])) : "memory");
}
__device__ __forceinline__ void tmem_st32(u32 taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
        "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])),
        "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Loads `n` (multiple of 8) consecutive f32 columns of this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void tmem_load_row(u32 taddr, float *v) {
  static_assert(N % 8 == 0, "TMEM row loads move multiples of 8 columns");
  int c = 0;
#pragma unroll
  for (; c + 32 <= N; c += 32) tmem_ld32(taddr + c, v + c);
#pragma unroll
  for (; c < N; c += 8) tmem_ld8(taddr + c, v + c);
  tmem_wait_ld();
}
template <int N>
__device__ __forceinline__ void tmem_store_row(u32 taddr, const float *v) {
  static_assert(N % 8 == 0, "TMEM row stores move multiples of 8 columns");
  int c = 0;
#pragma unroll
  for (; c + 32 <= N; c += 32) tmem_st32(taddr + c, v + c);
#pragma unroll
  for (; c < N; c += 8) tmem_st8(taddr + c, v + c);
  tmem_wait_st();
}
// The same stores without the wait: the caller issues tmem_wait_st() before
// anything reads these columns (an MMA operand read included).
template <int N>
__device__ __forceinline__ void tmem_store_row_async(u32 taddr, const float *v) {
  static_assert(N % 8 == 0, "TMEM row stores move multiples of 8 columns");
  int c = 0;
#pragma unroll
  for (; c + 32 <= N; c += 32) tmem_st32(taddr + c, v + c);
#pragma unroll
  for (; c < N; c += 8) tmem_st8(taddr + c, v + c);
}

// ---------------------------------------------------------------------------
// operand staging layouts for register-sourced MMA operands
// ---------------------------------------------------------------------------

// Byte offset of element (p, q) of a P x Q f16 operand stored K-major without
// swizzle: p indexes M (or N), q indexes K.  Core matrices are 8 rows x 16 B;
// the two core matrices of one K=16 step are LBO = 128 B apart and 8-row
// groups are SBO = Q * 16 B apart.
__device__ __forceinline__ u32 kmajor_offset(int p, int q, int Q) {
  return static_cast<u32>(((p >> 3) * (Q * 16)) + ((q >> 3) * 128) + ((p & 7) * 16) + ((q & 7) * 2));
}

}  // namespace tila
