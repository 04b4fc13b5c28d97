// The table of built-in kernel families a dispatch can name, with their
// argument signatures, the bounds checks run before any launch, and the
// launchers.

#include <cuda_runtime.h>

#include <climits>
#include <cstring>

#include "../mtl_internal.hpp"

namespace mtl {

int (*ew_emit_fn(const char* name))(const LaunchArgs&, std::vector<EwOp>&, int*, int*, int*);
mtl_status scatter_check(const LaunchArgs& la, const uint64_t* bytes);
uint64_t scatter_workspace(const LaunchArgs& la);
mtl_status scatter_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status fft_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status fft_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status gemm_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status gemm_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status conv_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status conv_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status nchwconv_check(const LaunchArgs& la, const uint64_t* bytes);
#define SC_DECL(k)                                               \
  mtl_status k##_check(const LaunchArgs& la, const uint64_t* bytes); \
  mtl_status k##_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
SC_DECL(sc_move_lights)
SC_DECL(sc_cull)
SC_DECL(sc_write_draw)
SC_DECL(sc_tile_lights)
SC_DECL(sc_ssao)
SC_DECL(sc_ao_blur)
SC_DECL(sc_shade)
SC_DECL(sc_bright)
SC_DECL(sc_blur)
SC_DECL(sc_composite)
#undef SC_DECL

mtl_status nchwconv_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status nhwc_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status nhwc_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status gapfc_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status gapfc_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
uint64_t gapfc_workspace(const LaunchArgs& la);
uint64_t conv_workspace(const LaunchArgs& la);
mtl_status advect_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status advect_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status clear_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status clear_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status splat_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status splat_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status pack_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status pack_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status unpack_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status unpack_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status blur_check(const LaunchArgs& la, const uint64_t* bytes);
mtl_status blur_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status scatter_dense_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
mtl_status raster_check(const LaunchArgs& la, const uint64_t* bytes);
uint64_t raster_workspace(const LaunchArgs& la);
mtl_status raster_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);
int gemm_timeouts(bool reset);
int conv_timeouts(bool reset);
int fft_timeouts(bool reset);
cudaError_t gemm_set_wait_limit(unsigned long long ns);
cudaError_t conv_set_wait_limit(unsigned long long ns);
void gemm_inject_stall(int launches);

// ── checks ──────────────────────────────────────────────────────────────────
static int64_t nd_total(const LaunchArgs& la) {
  int64_t t = 1;
  for (int i = 0; i < la.ndim; ++i) t *= la.nd[i];
  return t;
}

// Every buffer argument of an elementwise kernel is indexed 0..n-1.
static mtl_status check_elementwise(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = nd_total(la);
  for (size_t i = 0; i < la.a.size(); ++i) {
    if (la.a[i].kind != MTL_ARG_PTR) continue;
    if (bytes[i] && bytes[i] < (uint64_t)n * 4)
      return fail(MTL_ERR_ARGUMENT,
                  "elementwise kernel: buffer argument %zu has %llu bytes but the ndrange covers "
                  "%lld Float32 elements",
                  i + 1, (unsigned long long)bytes[i], (long long)n);
  }
  return MTL_OK;
}

// ── fill_span!(dst, base, v): dst[base + i] = v   test/test_window.jl:386-389 ─
__global__ void fill_span_kernel(float* dst, int64_t base, float v, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) dst[base + i] = v;
}
static mtl_status check_fill_span(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = nd_total(la);
  const int64_t base = la.a[1].i32;
  if (base < 0) return fail(MTL_ERR_ARGUMENT, "fill_span: negative base");
  if (bytes[0] && bytes[0] < (uint64_t)(base + n) * 4)
    return fail(MTL_ERR_ARGUMENT, "fill_span: writes elements %lld..%lld of a %llu-element buffer",
                (long long)base + 1, (long long)(base + n), (unsigned long long)(bytes[0] / 4));
  return MTL_OK;
}
static mtl_status run_fill_span(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = nd_total(la);
  if (n <= 0) return MTL_OK;
  int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)la.sm_count * 8);
  fill_span_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), la.a[1].i32, la.a[2].f32, n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "fill_span: %s", cudaGetErrorString(e));
}

// ── counters: bump_counter!(c) and clear_and_tally!(c, tally) ───────────────
// test/test_window.jl:334-341: every work item adds one to c[1] atomically;
// the clear writes 0 to c[1] and adds one to tally[1]. Warp-aggregated: one
// atomic per warp, with the warp's active count.
__global__ void bump_counter_kernel(uint32_t* c, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    unsigned mask = __activemask();
    int leader = __ffs(mask) - 1;
    if ((threadIdx.x & 31) == (unsigned)leader) atomicAdd(c, (uint32_t)__popc(mask));
  }
}
__global__ void clear_and_tally_kernel(uint32_t* c, uint32_t* tally) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    c[0] = 0;
    atomicAdd(tally, 1u);
  }
}
static mtl_status check_counter(const LaunchArgs& la, const uint64_t* bytes) {
  for (size_t i = 0; i < la.a.size(); ++i)
    if (la.a[i].kind == MTL_ARG_PTR && bytes[i] && bytes[i] < 4)
      return fail(MTL_ERR_ARGUMENT, "counter argument %zu is smaller than one UInt32", i + 1);
  return MTL_OK;
}
static mtl_status run_bump_counter(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = nd_total(la);
  if (n <= 0) return MTL_OK;
  int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)la.sm_count * 8);
  bump_counter_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<uint32_t*>(la.a[0].ptr), n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "bump_counter: %s", cudaGetErrorString(e));
}
static mtl_status run_clear_and_tally(const LaunchArgs& la, void*, uint64_t, void* stream) {
  clear_and_tally_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<uint32_t*>(la.a[0].ptr),
                                                              reinterpret_cast<uint32_t*>(la.a[1].ptr));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "clear_and_tally: %s", cudaGetErrorString(e));
}

// ── transpose_scale!(dst, src, w, h, a)   test/test_window.jl:30-33 ──────────
// Over the ndrange (nx, ny), 0-based: dst[ix*h + iy] = src[iy*w + ix] * a. The
// read runs along rows of src and the write down columns of it, so a block
// stages a 32 x 32 tile in shared memory (one column of padding: the column
// reads hit 32 different banks) and both global accesses are 128-byte rows.
constexpr int kTpTile = 32, kTpRows = 8;
__global__ void __launch_bounds__(kTpTile* kTpRows)
    transpose_scale_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t w, int64_t h, float a,
                           int64_t nx, int64_t ny) {
  __shared__ float tile[kTpTile][kTpTile + 1];
  const int64_t x0 = (int64_t)blockIdx.x * kTpTile, y0 = (int64_t)blockIdx.y * kTpTile;
#pragma unroll
  for (int r = threadIdx.y; r < kTpTile; r += kTpRows) {
    const int64_t ix = x0 + threadIdx.x, iy = y0 + r;
    if (ix < nx && iy < ny) tile[r][threadIdx.x] = __fmul_rn(src[iy * w + ix], a);
  }
  __syncthreads();
#pragma unroll
  for (int r = threadIdx.y; r < kTpTile; r += kTpRows) {
    const int64_t ix = x0 + r, iy = y0 + threadIdx.x;
    if (ix < nx && iy < ny) dst[ix * h + iy] = tile[threadIdx.x][r];
  }
}
static mtl_status check_transpose_scale(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 2) return fail(MTL_ERR_ARGUMENT, "transpose_scale: ndrange must be (w, h)");
  const int64_t w = la.a[2].i32, h = la.a[3].i32, nx = la.nd[0], ny = la.nd[1];
  if (w < 0 || h < 0 || nx > w || ny > h)
    return fail(MTL_ERR_ARGUMENT, "transpose_scale: ndrange (%lld, %lld) exceeds w = %lld, h = %lld", (long long)nx,
                (long long)ny, (long long)w, (long long)h);
  if (nx > 0 && ny > 0) {
    const uint64_t src_need = (uint64_t)((ny - 1) * w + nx) * 4, dst_need = (uint64_t)((nx - 1) * h + ny) * 4;
    if (bytes[1] && bytes[1] < src_need)
      return fail(MTL_ERR_ARGUMENT, "transpose_scale: src has %llu bytes, the launch reads %llu",
                  (unsigned long long)bytes[1], (unsigned long long)src_need);
    if (bytes[0] && bytes[0] < dst_need)
      return fail(MTL_ERR_ARGUMENT, "transpose_scale: dst has %llu bytes, the launch writes %llu",
                  (unsigned long long)bytes[0], (unsigned long long)dst_need);
  }
  return MTL_OK;
}
static mtl_status run_transpose_scale(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t nx = la.nd[0], ny = la.nd[1];
  if (nx <= 0 || ny <= 0) return MTL_OK;
  if ((nx + kTpTile - 1) / kTpTile > INT32_MAX || (ny + kTpTile - 1) / kTpTile > 65535)
    return fail(MTL_ERR_UNSUPPORTED, "transpose_scale: ndrange too large");
  dim3 grid((unsigned)((nx + kTpTile - 1) / kTpTile), (unsigned)((ny + kTpTile - 1) / kTpTile));
  transpose_scale_kernel<<<grid, dim3(kTpTile, kTpRows), 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), reinterpret_cast<const float*>(la.a[1].ptr), la.a[2].i32, la.a[3].i32,
      la.a[4].f32, nx, ny);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "transpose_scale: %s", cudaGetErrorString(e));
}

// ── frombytes!(dst, src): dst = Float32(src & 0xff)   test/test_window.jl:84-87
// 16-byte loads and stores when both pointers allow them.
__global__ void frombytes_kernel(float* __restrict__ dst, const uint32_t* __restrict__ src, int64_t n, bool vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t q = i; q < n4; q += stride) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + q);
      reinterpret_cast<float4*>(dst)[q] =
          make_float4((float)(v.x & 0xffu), (float)(v.y & 0xffu), (float)(v.z & 0xffu), (float)(v.w & 0xffu));
    }
    for (int64_t k = 4 * n4 + i; k < n; k += stride) dst[k] = (float)(src[k] & 0xffu);
  } else {
    for (int64_t k = i; k < n; k += stride) dst[k] = (float)(src[k] & 0xffu);
  }
}
static mtl_status run_frombytes(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = nd_total(la);
  if (n <= 0) return MTL_OK;
  const bool vec = ((la.a[0].ptr | la.a[1].ptr) & 15) == 0;
  const int64_t work = vec ? (n + 3) / 4 : n;
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)la.sm_count * 8);
  frombytes_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), reinterpret_cast<const uint32_t*>(la.a[1].ptr), n, vec);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "frombytes: %s", cudaGetErrorString(e));
}

// ── the table ───────────────────────────────────────────────────────────────
#define EW(name, sig, rd, wr) \
  { name, sig, true, rd, wr, check_elementwise, nullptr, nullptr, nullptr }

static KernelDesc g_kernels[] = {
    // reference kernels (bench/, test/)
    EW("stir", "BBf", 0b010, 0b001),
    EW("mix", "BBBf", 0b0110, 0b0001),
    EW("keep", "BB", 0b10, 0b01),
    EW("touch1", "B", 0b1, 0b1),
    EW("touch2", "BB", 0b11, 0b01),
    EW("touch3", "BBB", 0b111, 0b001),
    EW("touch4", "BBBB", 0b1111, 0b0001),
    EW("bump", "BBf", 0b010, 0b001),
    EW("scaleby", "BBf", 0b010, 0b001),
    EW("sched_write", "Bf", 0b00, 0b01),
    EW("sched_accum", "BB", 0b11, 0b01),
    // the elementwise chain workload, one op per kernel, and all eight at once
    EW("axpy", "BBBf", 0b0110, 0b0001),
    EW("mul", "BBB", 0b110, 0b001),
    EW("add", "BBB", 0b110, 0b001),
    EW("sub", "BBB", 0b110, 0b001),
    EW("fma", "BBBB", 0b1110, 0b0001),
    EW("abs", "BB", 0b10, 0b01),
    EW("sqrt_abs", "BB", 0b10, 0b01),
    EW("scale", "BBf", 0b010, 0b001),
    EW("chain8", "BBBB", 0b1110, 0b0001),
    {"fill_span", "Bif", false, 0b000, 0b001, check_fill_span, nullptr, run_fill_span, nullptr},
    // transpose_scale(dst, src, w, h, a) over the ndrange (w, h), 2-D
    {"transpose_scale", "BBiif", false, 0b00010, 0b00001, check_transpose_scale, nullptr, run_transpose_scale,
     nullptr},
    // frombytes(dst f32, src u32): the low byte as a float
    {"frombytes", "BB", false, 0b10, 0b01, check_elementwise, nullptr, run_frombytes, nullptr},
    {"bump_counter", "B", false, 0b1, 0b1, check_counter, nullptr, run_bump_counter, nullptr},
    {"clear_and_tally", "BB", false, 0b10, 0b11, check_counter, nullptr, run_clear_and_tally, nullptr},
    {"scatter_add", "bbbBii", false, 0b001100, 0b000011, scatter_check, scatter_workspace, scatter_run,
     nullptr},
    // the same arguments, for inputs whose bins pile up (warp-aggregated atomics)
    {"scatter_add_dense", "bbbBii", false, 0b001100, 0b000011, scatter_check, scatter_workspace,
     scatter_dense_run, nullptr},
    // batched complex FFT: out, in, length, inverse; ndrange = number of transforms
    {"fft_c2c", "BBii", false, 0b10, 0b01, fft_check, nullptr, fft_run, nullptr},
    // batched bf16 GEMM, fp32 accumulate and output: C, A, B, M, N, K; ndrange = batch
    {"gemm_bf16", "BBBiii", false, 0b110, 0b001, gemm_check, nullptr, gemm_run, nullptr},
    // NHWC bf16 convolution (implicit GEMM): out, in, w (HWIO), H, W, Cin, Cout,
    // k, stride, pad, relu, in_wpad, out_wpad; ndrange = images
    {"conv2d_bf16", "BBBiiiiiiiiii", false, 0b110, 0b001, conv_check, conv_workspace, conv_run, nullptr},
    // the first convolution straight from an NCHW input (C <= 4, stride 2):
    // out, in, w (HWIO, 4 input channels), H, W, C, Cout, k, stride, pad,
    // relu, out_wpad; ndrange = images
    {"conv2d_nchw_bf16", "BBBiiiiiiiii", false, 0b110, 0b001, nchwconv_check, nullptr, nchwconv_run, nullptr},
    // NCHW -> NHWC with zero-padded channels and Wpad zero columns each side:
    // out, in, C, H, W, Cpad, Wpad; ndrange = images
    {"nchw_to_nhwc_bf16", "BBiiiii", false, 0b10, 0b01, nhwc_check, nullptr, nhwc_run, nullptr},
    // global average pool + fully connected: logits, act, w, HW, C, classes; ndrange = images
    {"gap_fc", "BBBiii", false, 0b110, 0b001, gapfc_check, gapfc_workspace, gapfc_run, nullptr},
    // point clouds and image chains (bench/two_scatters.jl, bench/chain.jl), headless
    {"advect_points", "BBff", false, 0b11, 0b11, advect_check, nullptr, advect_run, nullptr},
    {"clear_rgba", "Bffff", false, 0b0, 0b1, clear_check, nullptr, clear_run, nullptr},
    {"splat_points", "BBBBBiiii", false, 0b11110, 0b00001, splat_check, nullptr, splat_run, nullptr},
    {"pack_bgra8", "BB", false, 0b10, 0b01, pack_check, nullptr, pack_run, nullptr},
    {"unpack_bgra8", "BBii", false, 0b10, 0b01, unpack_check, nullptr, unpack_run, nullptr},
    {"blur3x3", "BBii", false, 0b10, 0b01, blur_check, nullptr, blur_run, nullptr},
    // headless triangle rasterisation of instanced meshes (the g-buffer and shadow
    // passes of bench/showcase.jl and bench/deferred.jl): depth, out0..2, proto
    // positions, proto normals, visible, counter, centers, sizes, colors, params,
    // P, matrix offset, mode, W, H, vertices per instance; ndrange = instances
    {"raster_instances", "BbbbBbBBBBbbBiiiii", false, 0x1FF0, 0xF, raster_check, raster_workspace, raster_run,
     nullptr},
    // the showcase's compute passes (bench/showcase.jl), headless; P = scene constants
    {"sc_move_lights", "BBBBBBi", false, 0b0111110, 0b0000111, sc_move_lights_check, nullptr, sc_move_lights_run,
     nullptr},
    {"sc_cull", "BBBBi", false, 0b01110, 0b00011, sc_cull_check, nullptr, sc_cull_run, nullptr},
    {"sc_write_draw", "BBi", false, 0b010, 0b001, sc_write_draw_check, nullptr, sc_write_draw_run, nullptr},
    {"sc_tile_lights", "BBBBBiiiii", false, 0b0000011100, 0b0000000011, sc_tile_lights_check, nullptr,
     sc_tile_lights_run, nullptr},
    {"sc_ssao", "BBBBiii", false, 0b0001110, 0b0000001, sc_ssao_check, nullptr, sc_ssao_run, nullptr},
    {"sc_ao_blur", "BBB", false, 0b110, 0b001, sc_ao_blur_check, nullptr, sc_ao_blur_run, nullptr},
    {"sc_shade", "BBBBBBBBBBBBiii", false, 0b000111111111110, 0b000000000000001, sc_shade_check, nullptr,
     sc_shade_run, nullptr},
    {"sc_bright", "BBBiii", false, 0b000110, 0b000001, sc_bright_check, nullptr, sc_bright_run, nullptr},
    {"sc_blur", "BBii", false, 0b0010, 0b0001, sc_blur_check, nullptr, sc_blur_run, nullptr},
    {"sc_composite", "BBBBiii", false, 0b0001110, 0b0000001, sc_composite_check, nullptr, sc_composite_run,
     nullptr},
};
#undef EW

static bool g_init = false;
static void init_table() {
  if (g_init) return;
  for (KernelDesc& k : g_kernels)
    if (k.elementwise) k.ew_emit = ew_emit_fn(k.name);
  g_init = true;
}

const KernelDesc* kernel_desc(int id) {
  init_table();
  if (id < 0 || id >= (int)(sizeof g_kernels / sizeof g_kernels[0])) return nullptr;
  return &g_kernels[id];
}
int kernel_count() { return (int)(sizeof g_kernels / sizeof g_kernels[0]); }
int kernel_find(const char* name) {
  init_table();
  for (int i = 0; i < kernel_count(); ++i)
    if (!strcmp(g_kernels[i].name, name)) return i;
  return -1;
}

mtl_status launch_kernel(int kernel, const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  const KernelDesc* kd = kernel_desc(kernel);
  if (!kd) return fail(MTL_ERR_ARGUMENT, "unknown kernel %d", kernel);
  std::vector<uint64_t> bytes(la.a.size(), 0);
  for (size_t i = 0; i < la.a.size(); ++i) {
    bytes[i] = la.a[i].bytes;
    char c = kd->sig[i];
    if ((c == 'B') && (la.a[i].kind != MTL_ARG_PTR || la.a[i].ptr == 0))
      return fail(MTL_ERR_ARGUMENT, "%s: argument %zu must be a device buffer", kd->name, i + 1);
  }
  if (kd->check)
    if (mtl_status s = kd->check(la, bytes.data())) return s;
  if (kd->elementwise) return ew_launch_single(kd, la, stream);
  return kd->launch(la, ws, ws_bytes, stream);
}

}  // namespace mtl

extern "C" {

mtl_status mtl_kernel_lookup(const char* name, int32_t* kernel) {
  if (!name || !kernel) return mtl::fail(MTL_ERR_ARGUMENT, "mtl_kernel_lookup: NULL argument");
  int k = mtl::kernel_find(name);
  if (k < 0) return mtl::fail(MTL_ERR_ARGUMENT, "no built-in kernel named \"%s\"", name);
  *kernel = k;
  return MTL_OK;
}

mtl_status mtl_kernel_info(int32_t kernel, const char** name, const char** signature) {
  const mtl::KernelDesc* kd = mtl::kernel_desc(kernel);
  if (!kd) return mtl::fail(MTL_ERR_ARGUMENT, "unknown kernel %d", kernel);
  if (name) *name = kd->name;
  if (signature) *signature = kd->sig;
  return MTL_OK;
}

int32_t mtl_kernel_count(void) { return mtl::kernel_count(); }

mtl_status mtl_kernel_timeouts(int32_t reset, int64_t* count) {
  if (!count) return mtl::fail(MTL_ERR_ARGUMENT, "mtl_kernel_timeouts: NULL argument");
  int64_t total = 0;
  for (int v : {mtl::gemm_timeouts(reset != 0), mtl::conv_timeouts(reset != 0), mtl::fft_timeouts(reset != 0)}) {
    if (v < 0) return mtl::fail(MTL_ERR_CUDA, "mtl_kernel_timeouts: cannot read the device counters");
    total += v;
  }
  *count = total;
  return MTL_OK;
}

mtl_status mtl_set_wait_limit(uint64_t ns) {
  const uint64_t v = ns ? ns : 2000000000ull;
  if (v < 1000000ull) return mtl::fail(MTL_ERR_ARGUMENT, "mtl_set_wait_limit: %llu ns is below 1 ms", (unsigned long long)v);
  for (cudaError_t e : {mtl::gemm_set_wait_limit(v), mtl::conv_set_wait_limit(v)})
    if (e != cudaSuccess) return mtl::fail(MTL_ERR_CUDA, "mtl_set_wait_limit: %s", cudaGetErrorString(e));
  return MTL_OK;
}

mtl_status mtl_inject_stall(const char* kernel, int32_t launches) {
  if (!kernel) return mtl::fail(MTL_ERR_ARGUMENT, "mtl_inject_stall: NULL kernel name");
  if (std::strcmp(kernel, "gemm_bf16") != 0)
    return mtl::fail(MTL_ERR_UNSUPPORTED, "mtl_inject_stall: only gemm_bf16 has a stall hook, not %s", kernel);
  mtl::gemm_inject_stall(launches);
  return MTL_OK;
}

}  // extern "C"
