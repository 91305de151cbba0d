// extern "C" entry points of libspectra_b200.so (declared in
// include/spectra_b200.h).  Every argument check runs on the host before any
// CUDA call, so an invalid call returns a status code and launches nothing.
#include <cuda.h>

#include <cmath>
#include <cstring>
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "format.h"
#include "gemm.h"
#include "gemv.h"
#include "p2p.h"

namespace spectra {

namespace {
thread_local int g_last_cuda_error = 0;

bool is_float_dt(int dt) { return dt == SPECTRA_DT_F16 || dt == SPECTRA_DT_BF16 || dt == SPECTRA_DT_F32; }
bool is_index_dt(int dt) { return dt == SPECTRA_DT_I32 || dt == SPECTRA_DT_I64; }
size_t dt_size(int dt) { return (dt == SPECTRA_DT_F16 || dt == SPECTRA_DT_BF16) ? 2 : (dt == SPECTRA_DT_I64 ? 8 : 4); }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool fits_i32(int64_t v) { return v >= 0 && v <= INT32_MAX; }

// Shared checks of the quantised weight tensors.
int check_weights(const uint8_t* packed, const uint16_t* scales, const uint8_t* zeros,
                  int64_t N, int64_t K, int layout) {
  if (!packed || !scales || !zeros) return SPECTRA_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || (K % kGroup) != 0 || !fits_i32(N) || !fits_i32(K)) return SPECTRA_ERR_SHAPE;
  if (layout != SPECTRA_LAYOUT_MARLIN && layout != SPECTRA_LAYOUT_EVEN_ODD) return SPECTRA_ERR_UNSUPPORTED;
  if (!aligned(scales, 2)) return SPECTRA_ERR_ALIGNMENT;
  return SPECTRA_OK;
}
}  // namespace

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = int(e); }

namespace {
void* driver_entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return p;
}
}  // namespace

unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static const GetCurrent get_current = reinterpret_cast<GetCurrent>(driver_entry("cuCtxGetCurrent"));
  static const GetId get_id = reinterpret_cast<GetId>(driver_entry("cuCtxGetId"));
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECTRA_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool mma_path_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECTRA_B200_GEMV_MMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool pf_path_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECTRA_B200_GEMV_PF");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool sz_tma_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECTRA_B200_GEMM_SZ_TMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool pair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECTRA_B200_GEMM_PAIR");
    return v && v[0] == '1';
  }();
  return on;
}

}  // namespace spectra

using namespace spectra;

extern "C" {

int spectra_abi_version(void) { return SPECTRA_B200_ABI_VERSION; }

const char* spectra_status_string(int status) {
  switch (status) {
    case SPECTRA_OK: return "ok";
    case SPECTRA_ERR_NULL_POINTER: return "a required pointer is NULL";
    case SPECTRA_ERR_SHAPE: return "invalid shape (N, K > 0, K a multiple of 32, sizes within int32)";
    case SPECTRA_ERR_STRIDE: return "invalid stride";
    case SPECTRA_ERR_ALIGNMENT: return "pointer not aligned to its element size";
    case SPECTRA_ERR_DTYPE: return "unsupported dtype code";
    case SPECTRA_ERR_WORKSPACE: return "workspace missing or too small";
    case SPECTRA_ERR_CUDA: return "CUDA error (see spectra_last_cuda_error)";
    case SPECTRA_ERR_UNSUPPORTED: return "unsupported argument combination";
    default: return "unknown status";
  }
}

int spectra_last_cuda_error(void) { return g_last_cuda_error; }

int spectra_w4a16_gemv(
    const void* x, int x_dtype, int64_t x_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* bias, int bias_dtype,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* y, int y_dtype, int64_t y_stride,
    int64_t N, int64_t K, int layout, void* stream) {
  int st = check_weights(packed, scales, zeros, N, K, layout);
  if (st != SPECTRA_OK) return st;
  if (!x || !y) return SPECTRA_ERR_NULL_POINTER;
  if (!is_float_dt(x_dtype) || !is_float_dt(y_dtype)) return SPECTRA_ERR_DTYPE;
  if (bias && !is_float_dt(bias_dtype)) return SPECTRA_ERR_DTYPE;
  if (n_out < 0 || !fits_i32(n_out)) return SPECTRA_ERR_SHAPE;
  const bool has_out = n_out > 0 && outlier_idx && outlier_w;
  if (n_out > 0 && (!outlier_idx || !outlier_w)) return SPECTRA_ERR_NULL_POINTER;
  if (has_out && (!is_index_dt(idx_dtype) || !is_float_dt(ow_dtype))) return SPECTRA_ERR_DTYPE;
  if (y_stride == 0 && N > 1) return SPECTRA_ERR_STRIDE;
  if (!aligned(x, dt_size(x_dtype)) || !aligned(y, dt_size(y_dtype)) ||
      (bias && !aligned(bias, dt_size(bias_dtype))) ||
      (has_out && (!aligned(outlier_idx, dt_size(idx_dtype)) || !aligned(outlier_w, dt_size(ow_dtype)))))
    return SPECTRA_ERR_ALIGNMENT;
  GemvArgs a;
  a.x = x; a.x_dtype = x_dtype; a.x_stride = x_stride;
  a.packed = packed; a.w_rs = w_row_stride;
  a.scales = reinterpret_cast<const __half*>(scales); a.s_rs = s_row_stride; a.s_cs = s_col_stride;
  a.zeros = zeros; a.z_rs = z_row_stride; a.z_cs = z_col_stride;
  a.bias = bias; a.bias_dtype = bias_dtype;
  a.idx = has_out ? outlier_idx : nullptr; a.idx_dtype = idx_dtype; a.n_out = has_out ? int(n_out) : 0;
  a.ow = has_out ? outlier_w : nullptr; a.ow_dtype = ow_dtype; a.ow_rs = ow_row_stride; a.ow_cs = ow_col_stride;
  a.y = y; a.y_dtype = y_dtype; a.y_stride = y_stride;
  a.N = int(N); a.K = int(K); a.layout = layout;
  return launch_gemv(a, static_cast<cudaStream_t>(stream));
}

int spectra_w4a16_dequant(
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    void* out, int out_dtype, int64_t out_row_stride,
    int64_t N, int64_t K, int layout, void* stream) {
  int st = check_weights(packed, scales, zeros, N, K, layout);
  if (st != SPECTRA_OK) return st;
  if (!out) return SPECTRA_ERR_NULL_POINTER;
  if (!is_float_dt(out_dtype)) return SPECTRA_ERR_DTYPE;
  if (!aligned(out, dt_size(out_dtype))) return SPECTRA_ERR_ALIGNMENT;
  if (out_row_stride < K && N > 1) return SPECTRA_ERR_STRIDE;
  DequantArgs a;
  a.packed = packed; a.w_rs = w_row_stride;
  a.scales = reinterpret_cast<const __half*>(scales); a.s_rs = s_row_stride; a.s_cs = s_col_stride;
  a.zeros = zeros; a.z_rs = z_row_stride; a.z_cs = z_col_stride;
  a.out = out; a.out_dtype = out_dtype; a.out_rs = out_row_stride;
  a.N = N; a.K = int(K); a.layout = layout;
  return launch_dequant(a, static_cast<cudaStream_t>(stream));
}

int spectra_w4a16_gemm(
    const void* a, int a_dtype, int64_t a_row_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* c, int c_dtype, int64_t c_row_stride,
    int64_t M, int64_t N, int64_t K, int layout,
    void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_weights(packed, scales, zeros, N, K, layout);
  if (st != SPECTRA_OK) return st;
  if (!a || !c) return SPECTRA_ERR_NULL_POINTER;
  if (M <= 0 || !fits_i32(M) || int64_t(M) * N > INT32_MAX) return SPECTRA_ERR_SHAPE;
  if (a_dtype != SPECTRA_DT_F16 && a_dtype != SPECTRA_DT_BF16) return SPECTRA_ERR_DTYPE;
  if (c_dtype != a_dtype) return SPECTRA_ERR_DTYPE;
  if (n_out < 0 || !fits_i32(n_out)) return SPECTRA_ERR_SHAPE;
  const bool has_out = n_out > 0;
  if (has_out && (!outlier_idx || !outlier_w)) return SPECTRA_ERR_NULL_POINTER;
  if (has_out && (!is_index_dt(idx_dtype) || !is_float_dt(ow_dtype))) return SPECTRA_ERR_DTYPE;
  // tensor-map requirements (16-byte aligned bases and row strides)
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || (a_row_stride * 2) % 16 != 0 || a_row_stride < K)
    return SPECTRA_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || w_row_stride % 16 != 0 || w_row_stride < K / 2)
    return SPECTRA_ERR_ALIGNMENT;
  if (!aligned(c, 2) || (c_row_stride < N && M > 1)) return SPECTRA_ERR_STRIDE;
  if (has_out && (!aligned(outlier_idx, dt_size(idx_dtype)) || !aligned(outlier_w, dt_size(ow_dtype))))
    return SPECTRA_ERR_ALIGNMENT;
  GemmArgs g;
  g.a = a; g.a_dtype = a_dtype; g.a_rs = a_row_stride;
  g.packed = packed; g.w_rs = w_row_stride;
  g.scales = reinterpret_cast<const __half*>(scales); g.s_rs = s_row_stride; g.s_cs = s_col_stride;
  g.zeros = zeros; g.z_rs = z_row_stride; g.z_cs = z_col_stride;
  g.idx = has_out ? outlier_idx : nullptr; g.idx_dtype = idx_dtype; g.n_out = has_out ? int(n_out) : 0;
  g.ow = has_out ? outlier_w : nullptr; g.ow_dtype = ow_dtype; g.ow_rs = ow_row_stride; g.ow_cs = ow_col_stride;
  g.c = c; g.c_dtype = c_dtype; g.c_rs = c_row_stride;
  g.M = int(M); g.N = int(N); g.K = int(K); g.layout = layout;
  {  // the workspace contract does not depend on which kernel runs: checked first, on the host
    const GemmPlan pl = plan_gemm(M, N, K, n_out);
    if (pl.workspace > 0 && (workspace == nullptr || workspace_bytes < pl.workspace)) return SPECTRA_ERR_WORKSPACE;
  }
  if (M <= 16) {  // decode batch sizes: the raw-code small-M kernel when its layout conditions hold
    const int r = launch_gemv_mt(g, static_cast<cudaStream_t>(stream));
    if (r != SPECTRA_ERR_UNSUPPORTED) return r;
  }
  return launch_gemm(g, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int spectra_w4a16_gemm_noalloc(
    const void* a, int a_dtype, int64_t a_row_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* c, int c_dtype, int64_t c_row_stride,
    int64_t M, int64_t N, int64_t K, int layout, void* stream) {
  // the size limit is checked on the host before any CUDA call
  if (spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out) > size_t(SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES))
    return SPECTRA_ERR_WORKSPACE;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  const int st = gemm_noalloc_scratch(&scratch, &scratch_bytes);
  if (st != SPECTRA_OK) return st;
  return spectra_w4a16_gemm(a, a_dtype, a_row_stride, packed, w_row_stride, scales, s_row_stride, s_col_stride,
                            zeros, z_row_stride, z_col_stride, outlier_idx, idx_dtype, n_out, outlier_w, ow_dtype,
                            ow_row_stride, ow_col_stride, c, c_dtype, c_row_stride, M, N, K, layout, scratch,
                            scratch_bytes, stream);
}

int spectra_device_timeouts(int64_t* count, int reset) {
  if (!count) return SPECTRA_ERR_NULL_POINTER;
  long long a = 0, b = 0, c = 0, d = 0, e = 0;
  int st = gemv_timeouts(&a, reset != 0);
  if (st == SPECTRA_OK) st = gemv_pf_timeouts(&b, reset != 0);
  if (st == SPECTRA_OK) st = gemm_timeouts(&c, reset != 0);
  if (st == SPECTRA_OK) st = p2p_timeouts(&d, reset != 0);
  if (st == SPECTRA_OK) st = gemv_mt_timeouts(&e, reset != 0);
  if (st != SPECTRA_OK) return st;
  *count = int64_t(a + b + c + d + e);
  return SPECTRA_OK;
}

int64_t spectra_p2p_buffer_bytes(int64_t M, int64_t ns, int64_t elem_bytes, int world) {
  if (M < 1 || ns < 1 || world < 1 || world > kP2pMaxRanks || (elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8))
    return -1;
  if (M * ns * elem_bytes > (int64_t(1) << 34)) return -1;
  return p2p_buffer_bytes(int(M), int(ns), int(elem_bytes), world);
}

int spectra_p2p_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle) return SPECTRA_ERR_NULL_POINTER;
  if (bytes <= 0) return SPECTRA_ERR_SHAPE;
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, size_t(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, size_t(bytes));  // epoch slots start at 0
  if (e == cudaSuccess) e = cudaDeviceSynchronize();           // ... before any peer can see the handle
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return cuda_status(e);
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return SPECTRA_OK;
}

int spectra_p2p_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return SPECTRA_ERR_NULL_POINTER;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int spectra_p2p_close(void* ptr) {
  if (!ptr) return SPECTRA_ERR_NULL_POINTER;
  return cuda_status(cudaIpcCloseMemHandle(ptr));
}

int spectra_p2p_free(void* ptr) {
  if (!ptr) return SPECTRA_ERR_NULL_POINTER;
  return cuda_status(cudaFree(ptr));
}

int spectra_p2p_allgather(const void* src, void* const* peer_buffers, int64_t buffer_bytes, void* out,
                          int64_t out_row_stride, int64_t M, int64_t ns, int64_t N, int64_t elem_bytes, int* state,
                          int rank, int world, int64_t wait_limit_ns, void* stream) {
  if (!src || !peer_buffers || !out || !state) return SPECTRA_ERR_NULL_POINTER;
  if (world < 1 || world > kP2pMaxRanks || rank < 0 || rank >= world) return SPECTRA_ERR_SHAPE;
  if (M < 1 || ns < 1 || N < 1 || N > ns * world || wait_limit_ns <= 0)
    return SPECTRA_ERR_SHAPE;
  const int64_t need = spectra_p2p_buffer_bytes(M, ns, elem_bytes, world);
  if (need < 0) return elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8 ? SPECTRA_ERR_SHAPE : SPECTRA_ERR_DTYPE;
  if (buffer_bytes < need) return SPECTRA_ERR_WORKSPACE;
  if (out_row_stride < N || M * out_row_stride > (int64_t(1) << 34)) return SPECTRA_ERR_STRIDE;
  P2pArgs a{};
  for (int r = 0; r < world; ++r) {
    if (!peer_buffers[r]) return SPECTRA_ERR_NULL_POINTER;
    if (!aligned(peer_buffers[r], 16)) return SPECTRA_ERR_ALIGNMENT;
    a.peer[r] = static_cast<uint8_t*>(peer_buffers[r]);
  }
  if (!aligned(src, 16) || !aligned(out, size_t(elem_bytes)) || !aligned(state, 4)) return SPECTRA_ERR_ALIGNMENT;
  a.src = static_cast<const uint8_t*>(src);
  a.out = static_cast<uint8_t*>(out);
  a.out_rs = out_row_stride;
  a.slice_pitch = p2p_slice_pitch(int(M), int(ns), int(elem_bytes));
  a.state = state;
  a.M = int(M);
  a.ns = int(ns);
  a.N = int(N);
  a.elem_bytes = int(elem_bytes);
  a.rank = rank;
  a.world = world;
  a.wait_limit_ns = uint64_t(wait_limit_ns);
  return launch_p2p_allgather(a, static_cast<cudaStream_t>(stream));
}

int spectra_selftest_wait_timeout(void* stream) { return launch_selftest_wait(static_cast<cudaStream_t>(stream)); }

int spectra_quantize_group32(
    const void* w, int w_dtype, int64_t w_row_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    uint8_t* packed, int64_t p_row_stride,
    uint16_t* scales, int64_t s_row_stride,
    uint8_t* zeros, int64_t z_row_stride,
    uint8_t* packed_zeros, int64_t pz_row_stride,
    int64_t N, int64_t K, int layout, void* stream) {
  if (!w || !packed || !scales) return SPECTRA_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || K % kGroup != 0 || !fits_i32(N) || !fits_i32(K)) return SPECTRA_ERR_SHAPE;
  if (!is_float_dt(w_dtype)) return SPECTRA_ERR_DTYPE;
  if (layout != SPECTRA_LAYOUT_MARLIN && layout != SPECTRA_LAYOUT_EVEN_ODD) return SPECTRA_ERR_UNSUPPORTED;
  if (n_out < 0 || !fits_i32(n_out)) return SPECTRA_ERR_SHAPE;
  if (n_out > 0 && !outlier_idx) return SPECTRA_ERR_NULL_POINTER;
  if (n_out > 0 && !is_index_dt(idx_dtype)) return SPECTRA_ERR_DTYPE;
  const int64_t G = K / kGroup;
  if (w_row_stride < K || p_row_stride < K / 2 || s_row_stride < G || (zeros && z_row_stride < G) ||
      (packed_zeros && pz_row_stride < (G + 1) / 2))
    return SPECTRA_ERR_STRIDE;
  if (!aligned(w, dt_size(w_dtype)) || !aligned(scales, 2) || (n_out > 0 && !aligned(outlier_idx, dt_size(idx_dtype))))
    return SPECTRA_ERR_ALIGNMENT;
  QuantArgs a;
  a.w = w; a.w_dtype = w_dtype; a.w_rs = w_row_stride;
  a.idx = n_out > 0 ? outlier_idx : nullptr; a.idx_dtype = idx_dtype; a.n_out = int(n_out);
  a.packed = packed; a.p_rs = p_row_stride; a.packed_vec = aligned(packed, 16) && p_row_stride % 16 == 0;
  a.scales = scales; a.s_rs = s_row_stride;
  a.zeros = zeros; a.z_rs = z_row_stride;
  a.packed_zeros = packed_zeros; a.pz_rs = pz_row_stride;
  a.N = int(N); a.K = int(K); a.layout = layout;
  return launch_quantize_group32(a, static_cast<cudaStream_t>(stream));
}

int spectra_unpack_zeros(const uint8_t* packed_zeros, int64_t pz_row_stride, uint8_t* zeros, int64_t z_row_stride,
                         int64_t N, int64_t G, void* stream) {
  if (!packed_zeros || !zeros) return SPECTRA_ERR_NULL_POINTER;
  if (N <= 0 || G <= 0 || !fits_i32(G)) return SPECTRA_ERR_SHAPE;
  if (pz_row_stride < (G + 1) / 2 || z_row_stride < G) return SPECTRA_ERR_STRIDE;
  UnpackZerosArgs a;
  a.packed_zeros = packed_zeros; a.pz_rs = pz_row_stride;
  a.zeros = zeros; a.z_rs = z_row_stride;
  a.N = N; a.G = int(G);
  return launch_unpack_zeros(a, static_cast<cudaStream_t>(stream));
}

int spectra_kv_quantize(const void* t, int t_dtype, int64_t rows, int64_t D, uint8_t* packed, uint16_t* scales,
                        uint8_t* zeros, void* stream) {
  if (!t || !packed || !scales || !zeros) return SPECTRA_ERR_NULL_POINTER;
  if (rows < 0 || D <= 0 || !fits_i32(D)) return SPECTRA_ERR_SHAPE;
  if (t_dtype != SPECTRA_DT_BF16 && t_dtype != SPECTRA_DT_F16) return SPECTRA_ERR_DTYPE;
  if (!aligned(t, 2) || !aligned(packed, 16) || !aligned(scales, 2)) return SPECTRA_ERR_ALIGNMENT;
  if (rows == 0) return SPECTRA_OK;
  KvQuantArgs a;
  a.t = t; a.t_dtype = t_dtype; a.rows = rows; a.D = int(D);
  a.packed = packed; a.scales = scales; a.zeros = zeros;
  return launch_kv_quantize(a, static_cast<cudaStream_t>(stream));
}

int spectra_kv_dequantize(const uint8_t* packed, const uint16_t* scales, const uint8_t* zeros, void* out,
                          int out_dtype, int64_t rows, int64_t D, void* stream) {
  if (!packed || !scales || !zeros || !out) return SPECTRA_ERR_NULL_POINTER;
  if (rows < 0 || D <= 0 || !fits_i32(D)) return SPECTRA_ERR_SHAPE;
  if (!is_float_dt(out_dtype)) return SPECTRA_ERR_DTYPE;
  if (!aligned(packed, 16) || !aligned(scales, 2) || !aligned(out, dt_size(out_dtype))) return SPECTRA_ERR_ALIGNMENT;
  if (rows == 0) return SPECTRA_OK;
  KvDequantArgs a;
  a.packed = packed; a.scales = scales; a.zeros = zeros;
  a.out = out; a.out_dtype = out_dtype; a.rows = rows; a.D = int(D);
  return launch_kv_dequantize(a, static_cast<cudaStream_t>(stream));
}

int spectra_w4a16_embedding(
    const void* ids, int ids_dtype, int64_t T,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride,
    const uint8_t* zeros, int64_t z_row_stride, int zeros_packed,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride,
    void* out, int out_dtype, int64_t out_row_stride,
    int64_t V, int64_t K, int layout, void* stream) {
  if (!ids || !packed || !scales || !zeros || !out) return SPECTRA_ERR_NULL_POINTER;
  if (T < 0 || V <= 0 || K <= 0 || K % kGroup != 0 || !fits_i32(K)) return SPECTRA_ERR_SHAPE;
  if (!is_index_dt(ids_dtype) || !is_float_dt(out_dtype)) return SPECTRA_ERR_DTYPE;
  if (layout != SPECTRA_LAYOUT_MARLIN && layout != SPECTRA_LAYOUT_EVEN_ODD) return SPECTRA_ERR_UNSUPPORTED;
  if (n_out < 0 || !fits_i32(n_out)) return SPECTRA_ERR_SHAPE;
  if (n_out > 0 && (!outlier_idx || !outlier_w)) return SPECTRA_ERR_NULL_POINTER;
  if (n_out > 0 && (!is_index_dt(idx_dtype) || !is_float_dt(ow_dtype))) return SPECTRA_ERR_DTYPE;
  const int64_t G = K / kGroup;
  if (w_row_stride < K / 2 || s_row_stride < G || z_row_stride < (zeros_packed ? (G + 1) / 2 : G) ||
      out_row_stride < K || (n_out > 0 && ow_row_stride < n_out))
    return SPECTRA_ERR_STRIDE;
  if (!aligned(ids, dt_size(ids_dtype)) || !aligned(scales, 2) || !aligned(out, dt_size(out_dtype)) ||
      (n_out > 0 && (!aligned(outlier_idx, dt_size(idx_dtype)) || !aligned(outlier_w, dt_size(ow_dtype)))))
    return SPECTRA_ERR_ALIGNMENT;
  EmbedArgs a;
  a.ids = ids; a.ids_dtype = ids_dtype; a.T = T;
  a.packed = packed; a.w_rs = w_row_stride;
  a.scales = scales; a.s_rs = s_row_stride;
  a.zeros = zeros; a.z_rs = z_row_stride; a.zeros_packed = zeros_packed ? 1 : 0;
  a.idx = n_out > 0 ? outlier_idx : nullptr; a.idx_dtype = idx_dtype; a.n_out = int(n_out);
  a.ow = n_out > 0 ? outlier_w : nullptr; a.ow_dtype = ow_dtype; a.ow_rs = ow_row_stride;
  a.out = out; a.out_dtype = out_dtype; a.out_rs = out_row_stride;
  a.V = V; a.K = int(K); a.layout = layout;
  return launch_embedding(a, static_cast<cudaStream_t>(stream));
}

int spectra_argmax(const void* x, int x_dtype, int64_t x_row_stride, int64_t M, int64_t N, int64_t idx_offset,
                   int64_t* idx, float* val, void* stream) {
  if (!x || !idx) return SPECTRA_ERR_NULL_POINTER;
  if (M < 0 || N <= 0) return SPECTRA_ERR_SHAPE;
  if (!is_float_dt(x_dtype)) return SPECTRA_ERR_DTYPE;
  if (M > 1 && x_row_stride < N) return SPECTRA_ERR_STRIDE;
  if (!aligned(x, dt_size(x_dtype)) || !aligned(idx, 8) || (val && !aligned(val, 4))) return SPECTRA_ERR_ALIGNMENT;
  ArgmaxArgs a;
  a.x = x; a.x_dtype = x_dtype; a.x_rs = x_row_stride;
  a.idx = idx; a.val = val; a.M = M; a.N = N; a.idx_offset = idx_offset;
  return launch_argmax(a, static_cast<cudaStream_t>(stream));
}

int spectra_fwht(const void* x, int x_dtype, int64_t x_row_stride, void* y, int y_dtype, int64_t y_row_stride,
                 int64_t M, int64_t n, int normalize, void* stream) {
  if (!x || !y) return SPECTRA_ERR_NULL_POINTER;
  if (M < 0 || n <= 0 || n > 32768 || (n & (n - 1)) != 0) return SPECTRA_ERR_SHAPE;
  if (!is_float_dt(x_dtype) || !is_float_dt(y_dtype)) return SPECTRA_ERR_DTYPE;
  if (M > 1 && (x_row_stride < n || y_row_stride < n)) return SPECTRA_ERR_STRIDE;
  if (!aligned(x, dt_size(x_dtype)) || !aligned(y, dt_size(y_dtype))) return SPECTRA_ERR_ALIGNMENT;
  FwhtArgs a;
  a.x = x; a.x_dtype = x_dtype; a.x_rs = x_row_stride;
  a.y = y; a.y_dtype = y_dtype; a.y_rs = y_row_stride;
  a.M = M; a.n = int(n); a.normalize = normalize ? 1 : 0;
  a.inv_norm = float(std::sqrt(double(n)));  // the divisor, as the reference's res / math.sqrt(d)
  return launch_fwht(a, static_cast<cudaStream_t>(stream));
}

int spectra_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t n_out, int64_t* out) {
  if (!out) return SPECTRA_ERR_NULL_POINTER;
  if (M <= 0 || N <= 0 || K <= 0 || n_out < 0 || M > 2147483647LL || N > 2147483647LL || K > 2147483647LL)
    return SPECTRA_ERR_SHAPE;
  const GemmPlan pl = plan_gemm(M, N, K, n_out);
  out[0] = pl.MT; out[1] = pl.m_chunks; out[2] = pl.tiles_n; out[3] = pl.S; out[4] = pl.pair ? 1 : 0;
  out[5] = int64_t(pl.tiles_pad) * pl.S; out[6] = pl.act_stages; out[7] = int64_t(pl.workspace);
  return SPECTRA_OK;
}

int spectra_gemm_pair_capacity(int* clusters) {
  if (!clusters) return SPECTRA_ERR_NULL_POINTER;
  return gemm_pair_capacity(clusters);
}

size_t spectra_w4a16_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t n_out) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return plan_gemm(M, N, K, n_out).workspace;
}

}  // extern "C"
