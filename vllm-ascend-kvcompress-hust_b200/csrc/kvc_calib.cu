// Calibration reduction of pre-RoPE queries on sm_100a.
//
// Columns: a "rope unit" is (head, V consecutive frequencies) -- the thread
// reads V real parts q[f..f+V) and the matching V imaginary parts
// q[F+f..F+f+V) (16-byte vectors when V = 8) -- and a "pass unit" is (head, V
// consecutive unrotated dims).  The tokens are split into `rows` equal
// contiguous ranges (one per CTA row of the grid); each thread sums its column
// over its range in fp32 (|q| = sqrt(re^2 + im^2) per element) and writes that
// partial; a second kernel adds the partials in a fixed order in fp64 into the
// caller's running fp64 sums (atomics-free).  `rows` is at most one wave of
// resident CTAs and at most what the caller's workspace holds, so the fp32
// rounding -- and with it the last bits of the result -- is deterministic for a
// given device, workspace size and input, not across GPU models.
//
// Post-RoPE input (online calibration): the rotation of each row is undone in
// fp32 registers right after the load (theta = fp32(position) * omega_f, the
// product the rotary cache is built from), so the statistics see no extra
// rounding to the cache's 16-bit type.
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <mutex>

#include "kvc_common.cuh"

namespace kvc {

constexpr int kCalibChunk = 512;   // tokens per partial
constexpr int kCalibThreads = 256;

struct CalibArgs {
  const uint16_t* q;
  int64_t n_tok, row_stride;
  int H, D, F, P, V;
  int rope_cols, cols;
  double* ws;            // [rows][cols][3V]
  const float* omega;    // [F] for post-RoPE rows (positions first_pos + t), else null
  int64_t first_pos;
};

// |q| of one frequency pair (hardware square root: within 2 ulp of the
// correctly rounded value, far inside the statistics' tolerance)
__device__ __forceinline__ float modulus(float re, float im) {
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(fmaf(re, re, im * im)));
  return y;
}

template <int V, class E>
__device__ __forceinline__ void load_vals(const uint16_t* p, float (&x)[V]) {
  if constexpr (V == 8) {
    const uint4 v = ldg_stream16(p);
    x[0] = elem8<0>(v, E{}); x[1] = elem8<1>(v, E{}); x[2] = elem8<2>(v, E{}); x[3] = elem8<3>(v, E{});
    x[4] = elem8<4>(v, E{}); x[5] = elem8<5>(v, E{}); x[6] = elem8<6>(v, E{}); x[7] = elem8<7>(v, E{});
  } else if constexpr (V == 2) {
    const float2 t = unpack2(__ldg(reinterpret_cast<const uint32_t*>(p)), E{});
    x[0] = t.x; x[1] = t.y;
  } else {
    x[0] = unpack1(__ldg(p), E{});
  }
}

// Undo "half"-style RoPE of V frequency pairs of token position `pos` in fp32:
// the rotation was o1 = x1 cos - x2 sin, o2 = x2 cos + x1 sin.
template <int V>
__device__ __forceinline__ void unrotate_vals(float (&re)[V], float (&im)[V], const float* __restrict__ omega, int f,
                                              int64_t pos) {
#pragma unroll
  for (int j = 0; j < V; ++j) {
    float sn, cs;
    sincosf(__fmul_rn((float)pos, __ldg(omega + f + j)), &sn, &cs);
    const float o1 = re[j], o2 = im[j];
    re[j] = fmaf(o2, sn, o1 * cs);
    im[j] = fmaf(-o1, sn, o2 * cs);
  }
}

template <int V, class E, bool ROT>
__global__ void __launch_bounds__(1024) calib_partial_kernel(const __grid_constant__ CalibArgs a) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= a.cols) return;
  // balanced contiguous token ranges, one per CTA row (gridDim.y <= chunks)
  const int64_t span = (a.n_tok + gridDim.y - 1) / gridDim.y;
  const int64_t t0 = (int64_t)blockIdx.y * span;
  const int64_t t1 = min64(a.n_tok, t0 + span);
  double* out = a.ws + ((int64_t)blockIdx.y * a.cols + col) * 3 * V;
  if (col < a.rope_cols) {
    const int per = a.F / V;
    const int h = col / per, f = (col % per) * V;
    const uint16_t* base = a.q + (int64_t)h * a.D + f;
    float re[V], im[V], ab[V];
#pragma unroll
    for (int j = 0; j < V; ++j) re[j] = im[j] = ab[j] = 0.f;
    constexpr int U = 4;  // tokens whose loads are in flight together
    int64_t t = t0;
    for (; t + U <= t1; t += U) {
      float xr[U][V], xi[U][V];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        load_vals<V, E>(base + (t + u) * a.row_stride, xr[u]);
        load_vals<V, E>(base + (t + u) * a.row_stride + a.F, xi[u]);
      }
      if constexpr (ROT) {
#pragma unroll
        for (int u = 0; u < U; ++u) unrotate_vals<V>(xr[u], xi[u], a.omega, f, a.first_pos + t + u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int j = 0; j < V; ++j) {
          re[j] += xr[u][j];
          im[j] += xi[u][j];
          ab[j] += modulus(xr[u][j], xi[u][j]);
        }
    }
    for (; t < t1; ++t) {
      float xr[V], xi[V];
      load_vals<V, E>(base + t * a.row_stride, xr);
      load_vals<V, E>(base + t * a.row_stride + a.F, xi);
      if constexpr (ROT) unrotate_vals<V>(xr, xi, a.omega, f, a.first_pos + t);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        re[j] += xr[j];
        im[j] += xi[j];
        ab[j] += modulus(xr[j], xi[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < V; ++j) {
      out[j] = re[j];
      out[V + j] = im[j];
      out[2 * V + j] = ab[j];
    }
  } else {
    const int c = col - a.rope_cols;
    const int per = a.P / V;
    const int h = c / per, p = (c % per) * V;
    const uint16_t* base = a.q + (int64_t)h * a.D + 2 * a.F + p;
    float s[V];
#pragma unroll
    for (int j = 0; j < V; ++j) s[j] = 0.f;
    constexpr int U = 4;
    int64_t t = t0;
    for (; t + U <= t1; t += U) {
      float x[U][V];
#pragma unroll
      for (int u = 0; u < U; ++u) load_vals<V, E>(base + (t + u) * a.row_stride, x[u]);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int j = 0; j < V; ++j) s[j] += x[u][j];
    }
    for (; t < t1; ++t) {
      float x[V];
      load_vals<V, E>(base + t * a.row_stride, x);
#pragma unroll
      for (int j = 0; j < V; ++j) s[j] += x[j];
    }
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = s[j];
  }
}

// out element e of kind k (0 re, 1 im, 2 abs, 3 pass) <- sum over the partial
// rows: one warp per element, lanes take every 32nd row, fixed-order fp64
// shuffle tree (deterministic).
__global__ void __launch_bounds__(256) calib_finalize_kernel(const double* __restrict__ ws, int64_t nchunk, int cols,
                                                             int rope_cols, int H, int F, int P, int V,
                                                             double* re_sum, double* im_sum, double* abs_sum,
                                                             double* pass_sum) {
  const int64_t rope_elems = (int64_t)H * F;
  const int64_t total = 3 * rope_elems + (int64_t)H * P;
  const int64_t e = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (e >= total) return;
  int col, slot;
  double* dst;
  if (e < 3 * rope_elems) {
    const int kind = (int)(e / rope_elems);
    const int64_t i = e % rope_elems;  // h*F + f
    const int h = (int)(i / F), f = (int)(i % F);
    col = h * (F / V) + f / V;
    slot = kind * V + f % V;
    dst = (kind == 0 ? re_sum : kind == 1 ? im_sum : abs_sum) + i;
  } else {
    const int64_t i = e - 3 * rope_elems;  // h*P + p
    const int h = (int)(i / P), p = (int)(i % P);
    col = rope_cols + h * (P / V) + p / V;
    slot = p % V;
    dst = pass_sum + i;
  }
  double acc = 0.0;
  for (int64_t c = lane; c < nchunk; c += 32) acc += ws[((int64_t)c * cols + col) * 3 * V + slot];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) *dst += acc;
}

inline int calib_vec(int F, int P, int64_t row_stride, const void* q) {
  if (F % 8 == 0 && P % 8 == 0 && row_stride % 8 == 0 && aligned(q, 16)) return 8;
  if (F % 2 == 0 && P % 2 == 0 && row_stride % 2 == 0 && aligned(q, 4)) return 2;
  return 1;
}

}  // namespace kvc

using namespace kvc;

// Undo "half"-style (NeoX) RoPE in place: with theta = fp32(position) * omega_f
// (the fp32 product the rotary cache is built from) the rotation was
//   o1 = x1 cos - x2 sin,  o2 = x2 cos + x1 sin   (x1 = q[f], x2 = q[F + f]),
// so x1 = o1 cos + o2 sin, x2 = o2 cos - o1 sin.  One thread per (token, f):
// it forms the angle once and applies it to every head.
template <class E>
__global__ void unrotate_kernel(uint16_t* q, int64_t n_tok, int64_t row_stride, int heads, int D, int F,
                                int64_t first_pos, const float* __restrict__ omega) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tok * F) return;
  const int64_t t = i / F;
  const int f = (int)(i - t * F);
  const float theta = __fmul_rn((float)(first_pos + t), __ldg(omega + f));
  float sn, cs;
  sincosf(theta, &sn, &cs);
  uint16_t* row = q + t * row_stride;
  for (int h = 0; h < heads; ++h) {
    uint16_t* x = row + (int64_t)h * D;
    const float o1 = unpack1(x[f], E{}), o2 = unpack1(x[F + f], E{});
    const float x1 = fmaf(o2, sn, o1 * cs);
    const float x2 = fmaf(-o1, sn, o2 * cs);
    x[f] = pack1(x1, E{});
    x[F + f] = pack1(x2, E{});
  }
}

extern "C" int kvc_unrotate_queries(void* q, int dtype, int64_t n_tokens, int64_t row_stride, int heads,
                                    int head_dim, int rotary_dim, int64_t first_position, const float* omega,
                                    void* stream) {
  KVC_CHECK_ARG(q && omega, KVC_ENULL);
  KVC_CHECK_ARG(dtype == KVC_BF16 || dtype == KVC_FP16, KVC_EINVAL);
  KVC_CHECK_ARG(n_tokens >= 0 && heads > 0 && head_dim > 0 && rotary_dim > 0 && rotary_dim % 2 == 0 &&
                    rotary_dim <= head_dim && first_position >= 0 && row_stride >= (int64_t)heads * head_dim,
                KVC_EINVAL);
  KVC_CHECK_ARG(aligned(q, 2), KVC_EALIGN);
  if (n_tokens == 0) return KVC_OK;
  const int F = rotary_dim / 2;
  const int64_t work = n_tokens * F;
  const unsigned grid = (unsigned)((work + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == KVC_BF16)
    unrotate_kernel<Bf16><<<grid, 256, 0, st>>>((uint16_t*)q, n_tokens, row_stride, heads, head_dim, F,
                                                 first_position, omega);
  else
    unrotate_kernel<Fp16><<<grid, 256, 0, st>>>((uint16_t*)q, n_tokens, row_stride, heads, head_dim, F,
                                                 first_position, omega);
  return launch_status();
}

namespace kvc {

// Doubles of one partial row: every column writes 3V doubles (re, im, |.| or
// V pass sums), i.e. 3 * heads * (F + P) whatever the vector width V.
inline int64_t calib_row_doubles(int H, int F, int P) { return 3LL * H * (F + P); }

struct CalibPlan {
  int V, rope_cols, cols, threads, gx;
  int64_t rows;  // partial rows = CTA rows of the grid
};

// Launch shape for n tokens at vector width V: one CTA spans all columns of a
// token range where possible; the rows are at most ceil(n / kCalibChunk) and at
// most one full wave of resident CTAs (no tail wave), and at most `max_rows`.
inline CalibPlan calib_plan(int64_t n, int H, int F, int P, int V, int64_t max_rows) {
  CalibPlan c{};
  c.V = V;
  c.rope_cols = H * (F / V);
  c.cols = c.rope_cols + H * (P / V);
  c.threads = std::min(1024, (c.cols + 31) / 32 * 32);
  c.gx = (c.cols + c.threads - 1) / c.threads;
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, calib_partial_kernel<8, Bf16, false>, c.threads, 0) !=
          cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t wave = std::max<int64_t>(1, (int64_t)sm_count() * per_sm / c.gx);
  c.rows = std::min<int64_t>({(n + kCalibChunk - 1) / kCalibChunk, wave, max_rows, 65535});
  c.rows = std::max<int64_t>(c.rows, 1);
  return c;
}

// Shared body of the calibration entry points (arguments validated by the caller).
int calib_launch(const void* q, int dtype, int64_t n_tokens, int64_t row_stride, int heads, int head_dim,
                 int rotary_dim, double* re_sum, double* im_sum, double* abs_sum, double* pass_sum, double* ws,
                 int64_t ws_doubles, const float* omega, int64_t first_pos, cudaStream_t st) {
  const int F = rotary_dim / 2, P = head_dim - rotary_dim;
  const int64_t max_rows = ws_doubles / calib_row_doubles(heads, F, P);
  KVC_CHECK_ARG(max_rows >= 1, KVC_EINVAL);
  const CalibPlan c = calib_plan(n_tokens, heads, F, P, calib_vec(F, P, row_stride, q), max_rows);
  CalibArgs a{};
  a.q = (const uint16_t*)q;
  a.n_tok = n_tokens;
  a.row_stride = row_stride;
  a.H = heads;
  a.D = head_dim;
  a.F = F;
  a.P = P;
  a.V = c.V;
  a.rope_cols = c.rope_cols;
  a.cols = c.cols;
  a.ws = ws;
  a.omega = omega;
  a.first_pos = first_pos;
  const dim3 grid(c.gx, (unsigned)c.rows);
#define KVC_CALIB(VV, EE)                                                                  \
  (omega ? calib_partial_kernel<VV, EE, true><<<grid, c.threads, 0, st>>>(a)               \
         : calib_partial_kernel<VV, EE, false><<<grid, c.threads, 0, st>>>(a))
  if (dtype == KVC_BF16) {
    if (c.V == 8) KVC_CALIB(8, Bf16); else if (c.V == 2) KVC_CALIB(2, Bf16); else KVC_CALIB(1, Bf16);
  } else {
    if (c.V == 8) KVC_CALIB(8, Fp16); else if (c.V == 2) KVC_CALIB(2, Fp16); else KVC_CALIB(1, Fp16);
  }
#undef KVC_CALIB
  int rc = launch_status();
  if (rc != KVC_OK) return rc;
  const int64_t total = 3LL * heads * F + (int64_t)heads * P;
  calib_finalize_kernel<<<(unsigned)((total * 32 + 255) / 256), 256, 0, st>>>(
      ws, c.rows, c.cols, c.rope_cols, heads, F, P, c.V, re_sum, im_sum, abs_sum, pass_sum);
  return launch_status();
}

inline int calib_check(const void* q, int dtype, int64_t n_tokens, int64_t row_stride, int heads, int head_dim,
                       int rotary_dim, const double* re_sum, const double* im_sum, const double* abs_sum,
                       const double* pass_sum) {
  KVC_CHECK_ARG(q && re_sum && im_sum && abs_sum, KVC_ENULL);
  KVC_CHECK_ARG(dtype == KVC_BF16 || dtype == KVC_FP16, KVC_EINVAL);
  KVC_CHECK_ARG(n_tokens >= 0 && heads > 0 && head_dim > 0 && rotary_dim > 0 && rotary_dim <= head_dim &&
                    rotary_dim % 2 == 0 && row_stride >= (int64_t)heads * head_dim,
                KVC_EINVAL);
  KVC_CHECK_ARG(rotary_dim == head_dim || pass_sum != nullptr, KVC_ENULL);
  KVC_CHECK_ARG(aligned(q, 2), KVC_EALIGN);
  return KVC_OK;
}

}  // namespace kvc

extern "C" int64_t kvc_calibration_workspace_doubles(int64_t n_tokens, int heads, int head_dim, int rotary_dim) {
  if (n_tokens <= 0 || heads <= 0 || head_dim <= 0 || rotary_dim <= 0 || rotary_dim > head_dim) return 0;
  const int F = rotary_dim / 2, P = head_dim - rotary_dim;
  // the largest row count any vector width can plan (the width depends on the
  // caller's pointer and stride alignment)
  int64_t rows = 1;
  for (int V : {1, 2, 8})
    if (F % V == 0 && P % V == 0) rows = std::max(rows, calib_plan(n_tokens, heads, F, P, V, INT64_MAX).rows);
  return rows * calib_row_doubles(heads, F, P);
}

extern "C" int kvc_calibration_accumulate(const void* q, int dtype, int64_t n_tokens, int64_t row_stride, int heads,
                                          int head_dim, int rotary_dim, double* re_sum, double* im_sum,
                                          double* abs_sum, double* pass_sum, double* workspace,
                                          int64_t workspace_doubles, void* stream) {
  const int rc = calib_check(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum,
                             pass_sum);
  if (rc != KVC_OK) return rc;
  KVC_CHECK_ARG(workspace, KVC_ENULL);
  if (n_tokens == 0) return KVC_OK;
  return calib_launch(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum, pass_sum,
                      workspace, workspace_doubles, nullptr, 0, (cudaStream_t)stream);
}

extern "C" int kvc_calibration_accumulate_post_rope(const void* q, int dtype, int64_t n_tokens, int64_t row_stride,
                                                    int heads, int head_dim, int rotary_dim, int64_t first_position,
                                                    const float* omega, double* re_sum, double* im_sum,
                                                    double* abs_sum, double* pass_sum, double* workspace,
                                                    int64_t workspace_doubles, void* stream) {
  const int rc = calib_check(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum,
                             pass_sum);
  if (rc != KVC_OK) return rc;
  KVC_CHECK_ARG(workspace && omega, KVC_ENULL);
  KVC_CHECK_ARG(first_position >= 0, KVC_EINVAL);
  if (n_tokens == 0) return KVC_OK;
  return calib_launch(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum, pass_sum,
                      workspace, workspace_doubles, omega, first_position, (cudaStream_t)stream);
}

namespace kvc {

// ---------------------------------------------------------------------------
// Allocation-free variant: chunk partials in library-owned static device memory
// ---------------------------------------------------------------------------
//
// Some hosts cannot hand this library a device workspace: a process whose GPU
// memory was reserved up front (vLLM sizes the KV cache to fill the memory
// budget, so a later cudaMalloc can fail), or a foreign-language host that binds
// only this C ABI and has no device allocator.  For them the partial rows of
// the calibration reduction live in one file-scope __device__ array that every
// GPU loading the library keeps until process exit.  The launch plans only as
// many partial rows as the array holds (each thread then sums a longer token
// range), so the token count is not limited; only a head geometry whose single
// row exceeds the array is refused.  The array is shared by all calls on a
// device: calls that overlap on the GPU (different streams or threads without
// ordering) race on it.  Nothing in it must start at zero: each call writes
// every partial it later reads.

static __device__ __align__(256) double g_calib_scratch[KVC_CALIB_STATIC_SCRATCH_DOUBLES];

namespace {

constexpr int kMaxDevices = 64;

PFN_cuCtxGetCurrent_v4000 ctx_current_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }
  return fn;
}

// Device address of g_calib_scratch on the current device (host code must not
// use the symbol's name as a device pointer).  Resolved on the first call per
// device and again whenever the device's current context changes (a
// cudaDeviceReset reloads the module, so an address cached before it would be
// stale).
int static_scratch(double** out) {
  static std::mutex mu;
  static double* ptrs[kMaxDevices] = {};
  static CUcontext ctxs[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KVC_ECUDA;
  std::lock_guard<std::mutex> lock(mu);
  CUcontext ctx = nullptr;
  if (ptrs[dev] != nullptr) {
    PFN_cuCtxGetCurrent_v4000 cur = ctx_current_fn();
    if (cur == nullptr || cur(&ctx) != CUDA_SUCCESS || ctx != ctxs[dev]) ptrs[dev] = nullptr;
  }
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_calib_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return KVC_ECUDA;
    }
    PFN_cuCtxGetCurrent_v4000 cur = ctx_current_fn();
    ctx = nullptr;
    if (cur != nullptr) cur(&ctx);
    ptrs[dev] = static_cast<double*>(p);
    ctxs[dev] = ctx;
  }
  *out = ptrs[dev];
  return KVC_OK;
}

}  // namespace
}  // namespace kvc

extern "C" int kvc_calibration_accumulate_noalloc(const void* q, int dtype, int64_t n_tokens, int64_t row_stride,
                                                  int heads, int head_dim, int rotary_dim, double* re_sum,
                                                  double* im_sum, double* abs_sum, double* pass_sum, void* stream) {
  int rc = calib_check(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum,
                       pass_sum);
  if (rc != KVC_OK) return rc;
  const int F = rotary_dim / 2, P = head_dim - rotary_dim;
  if (calib_row_doubles(heads, F, P) > KVC_CALIB_STATIC_SCRATCH_DOUBLES) return KVC_ECAPACITY;
  if (n_tokens == 0) return KVC_OK;
  double* scratch = nullptr;
  rc = kvc::static_scratch(&scratch);
  if (rc != KVC_OK) return rc;
  return calib_launch(q, dtype, n_tokens, row_stride, heads, head_dim, rotary_dim, re_sum, im_sum, abs_sum, pass_sum,
                      scratch, KVC_CALIB_STATIC_SCRATCH_DOUBLES, nullptr, 0, (cudaStream_t)stream);
}
