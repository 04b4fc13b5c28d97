// Fused elementwise runs compiled to straight-line kernels when a plan is
// built — the counterpart of the reference's Pipelines phase, which compiles
// each dispatch's kernel at Plan time (ext/MantleLavaExt.jl:1832-1934), never
// per frame.
//
// A fused run's micro-op program (kernels/elementwise.cu) is printed as CUDA
// C++: one __global__ function whose body is the program's ops as plain
// statements on scalar registers, applied to the four lanes of each 128-bit
// load. It is compiled with NVRTC for sm_100a straight to a cubin (no PTX is
// read or kept), loaded with cudaLibraryLoadData and cached by its source
// text, so a plan rebuilt with the same chain reuses the kernel. The
// statements use the same round-to-nearest intrinsics as the interpreter, so
// results are bit-identical to it and to the oracle.
//
// NVRTC is opened with dlopen; where it is missing, or a pointer is not 16-byte
// aligned, the run keeps the interpreter kernel.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../mtl_internal.hpp"

namespace mtl {

namespace {
struct Nvrtc {
  void* h = nullptr;
  nvrtcResult (*Create)(nvrtcProgram*, const char*, const char*, int, const char* const*, const char* const*) = nullptr;
  nvrtcResult (*Compile)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*LogSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*Log)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*CubinSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*Cubin)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*Destroy)(nvrtcProgram*) = nullptr;
  bool tried = false;
};
Nvrtc g_rtc;
std::mutex g_rtc_mu;
std::map<std::string, cudaKernel_t> g_compiled;

bool load_nvrtc() {
  if (g_rtc.tried) return g_rtc.h != nullptr;
  g_rtc.tried = true;
  void* h = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnvrtc.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) return false;
#define SYM(f, n)                           \
  *(void**)(&g_rtc.f) = dlsym(h, n);        \
  if (!g_rtc.f) {                           \
    dlclose(h);                             \
    return false;                           \
  }
  SYM(Create, "nvrtcCreateProgram");
  SYM(Compile, "nvrtcCompileProgram");
  SYM(LogSize, "nvrtcGetProgramLogSize");
  SYM(Log, "nvrtcGetProgramLog");
  SYM(CubinSize, "nvrtcGetCUBINSize");
  SYM(Cubin, "nvrtcGetCUBIN");
  SYM(Destroy, "nvrtcDestroyProgram");
#undef SYM
  g_rtc.h = h;
  return true;
}

std::string reg(int r) { return "r" + std::to_string(r); }

std::string imm(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  char buf[40];
  snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", u);
  return buf;
}

std::string op_expr(const EwOp& o) {
  const std::string a = reg(o.a), b = reg(o.b), c = reg(o.c);
  switch (o.op) {
    case EW_MOV: return a;
    case EW_ADD: return "__fadd_rn(" + a + ", " + b + ")";
    case EW_SUB: return "__fsub_rn(" + a + ", " + b + ")";
    case EW_MUL: return "__fmul_rn(" + a + ", " + b + ")";
    case EW_FMA: return "__fmaf_rn(" + a + ", " + b + ", " + c + ")";
    case EW_ABS: return "fabsf(" + a + ")";
    case EW_SQRT: return "__fsqrt_rn(" + a + ")";
    case EW_SIN: return "sinf(" + a + ")";
    case EW_MULK: return "__fmul_rn(" + a + ", " + imm(o.imm) + ")";
    case EW_ADDK: return "__fadd_rn(" + a + ", " + imm(o.imm) + ")";
    default: return imm(o.imm);
  }
}

std::string source(const EwProgram& p) {
  const int nin = (int)p.inputs.size(), nout = (int)p.outputs.size();
  std::string params;
  for (int i = 0; i < nin; ++i) params += "const float* __restrict__ in" + std::to_string(i) + ", ";
  for (int j = 0; j < nout; ++j) params += "float* __restrict__ out" + std::to_string(j) + ", ";
  // elem(): the program on one element. Registers r0..r(nin-1) start as the
  // inputs; the ops are the program's, in order; outputs are read at the end.
  std::string loads;
  for (int i = 0; i < nin; ++i) loads += "  " + reg(i) + " = x" + std::to_string(i) + ";\n";
  std::string decls, ops;
  for (int r = 0; r < p.nregs; ++r) decls += "  float " + reg(r) + " = 0.f; (void)" + reg(r) + ";\n";
  for (const EwOp& o : p.ops) ops += "  " + reg(o.dst) + " = " + op_expr(o) + ";\n";
  std::string stores;
  for (int j = 0; j < nout; ++j) stores += "  y" + std::to_string(j) + " = " + reg(p.out_regs[j]) + ";\n";
  std::string fn = "__device__ __forceinline__ void elem(";
  for (int i = 0; i < nin; ++i) fn += "float x" + std::to_string(i) + ", ";
  for (int j = 0; j < nout; ++j) fn += std::string(j ? ", " : "") + "float& y" + std::to_string(j);
  fn += ") {\n" + decls + loads + ops + stores + "}\n";

  std::string k = fn + "extern \"C\" __global__ void __launch_bounds__(256) mtl_fused(" + params + "long long n) {\n";
  k += "  const long long groups = n >> 2;\n";
  k += "  const long long stride = (long long)gridDim.x * blockDim.x;\n";
  // Two groups per thread per iteration (g and g + stride): every load of
  // both is issued before any arithmetic, so twice the bytes are in flight.
  // Loads and stores carry the streaming (evict-first) hint: each byte is
  // touched once a replay (measured on B200, the eight-op chain at 2^22 over
  // four copies in turn: 13.6 us a step against 14.0 with default caching;
  // the hint on the stores alone 14.3, on the loads alone 13.9).
  auto group = [&](const std::string& gi, const std::string& tag) {
    std::string t;
    for (int i = 0; i < nin; ++i)
      t += "      const float4 v" + tag + std::to_string(i) + " = __ldcs(reinterpret_cast<const float4*>(in" +
           std::to_string(i) + ") + " + gi + ");\n";
    return t;
  };
  auto apply = [&](const std::string& gi, const std::string& tag) {
    std::string t;
    for (int j = 0; j < nout; ++j) t += "      float4 w" + tag + std::to_string(j) + ";\n";
    for (const char* lane : {"x", "y", "z", "w"}) {
      t += "      elem(";
      for (int i = 0; i < nin; ++i) t += "v" + tag + std::to_string(i) + "." + lane + ", ";
      for (int j = 0; j < nout; ++j) t += std::string(j ? ", " : "") + "w" + tag + std::to_string(j) + "." + lane;
      t += ");\n";
    }
    for (int j = 0; j < nout; ++j)
      t += "      __stcs(reinterpret_cast<float4*>(out" + std::to_string(j) + ") + " + gi + ", w" + tag + std::to_string(j) +
           ");\n";
    return t;
  };
  // programmatic dependent launch: wait for the previous grid's memory, then
  // let the next kernel's CTAs take SMs as this grid's finish
  k += "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  k += "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
  k += "  long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;\n";
  k += "  for (; g + stride < groups; g += 2 * stride) {\n";
  k += "    {\n" + group("g", "a") + group("g + stride", "b") + apply("g", "a") + apply("g + stride", "b") +
       "    }\n";
  k += "  }\n";
  k += "  if (g < groups) {\n" + group("g", "a") + apply("g", "a") + "  }\n";
  // the ragged tail (at most three elements), one per thread of block 0
  k += "  const long long t = (groups << 2) + threadIdx.x;\n";
  k += "  if (blockIdx.x == 0 && t < n) {\n";
  for (int j = 0; j < nout; ++j) k += "    float y" + std::to_string(j) + ";\n";
  k += "    elem(";
  for (int i = 0; i < nin; ++i) k += "in" + std::to_string(i) + "[t], ";
  for (int j = 0; j < nout; ++j) k += std::string(j ? ", " : "") + "y" + std::to_string(j);
  k += ");\n";
  for (int j = 0; j < nout; ++j) k += "    out" + std::to_string(j) + "[t] = y" + std::to_string(j) + ";\n";
  k += "  }\n}\n";
  return k;
}
}  // namespace

// Compile (or find) the straight-line kernel of a program. Returns MTL_OK with
// *kernel set; MTL_ERR_UNSUPPORTED when NVRTC is not on this machine (the
// caller then keeps the interpreter); any other failure is an error. Makes no
// stream operation: call it outside stream capture.
mtl_status ew_compile(const EwProgram& p, void** kernel) {
  *kernel = nullptr;
  if (p.outputs.empty()) return fail(MTL_ERR_UNSUPPORTED, "nothing to compile");
  const std::string src = source(p);
  std::lock_guard<std::mutex> lk(g_rtc_mu);
  auto it = g_compiled.find(src);
  if (it != g_compiled.end()) {
    *kernel = (void*)it->second;
    return MTL_OK;
  }
  if (!load_nvrtc()) return fail(MTL_ERR_UNSUPPORTED, "NVRTC is not available");
  nvrtcProgram prog;
  if (g_rtc.Create(&prog, src.c_str(), "mtl_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return fail(MTL_ERR_CUDA, "NVRTC: cannot create the program");
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17"};
  nvrtcResult r = g_rtc.Compile(prog, 2, opts);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    g_rtc.LogSize(prog, &n);
    std::string log(n, '\0');
    if (n) g_rtc.Log(prog, &log[0]);
    g_rtc.Destroy(&prog);
    return fail(MTL_ERR_CUDA, "NVRTC could not compile a fused run: %s", log.c_str());
  }
  size_t n = 0;
  g_rtc.CubinSize(prog, &n);
  std::string cubin(n, '\0');
  g_rtc.Cubin(prog, &cubin[0]);
  g_rtc.Destroy(&prog);
  cudaLibrary_t lib = nullptr;
  cudaError_t e = cudaLibraryLoadData(&lib, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
  cudaKernel_t k = nullptr;
  if (e == cudaSuccess) e = cudaLibraryGetKernel(&k, lib, "mtl_fused");
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MTL_ERR_CUDA, "loading a compiled fused run: %s", cudaGetErrorString(e));
  }
  g_compiled[src] = k;  // libraries stay loaded for the process: plans may share them
  *kernel = (void*)k;
  return MTL_OK;
}

// Launch a compiled program (pointers must be 16-byte aligned).
mtl_status ew_launch_compiled(void* kernel, const EwProgram& p, void* stream) {
  const int nin = (int)p.inputs.size(), nout = (int)p.outputs.size();
  constexpr int kMaxPtrs = 32;  // well above what ew_program_fits lets through
  if (nin + nout > kMaxPtrs) return fail(MTL_ERR_UNSUPPORTED, "compiled fused run: too many arguments");
  // no allocation and no attribute query per launch: a one-kernel plan issues
  // this for every run!
  void* args[kMaxPtrs + 1];
  uint64_t ptrs[kMaxPtrs];
  for (int i = 0; i < nin; ++i) ptrs[i] = p.inputs[i];
  for (int j = 0; j < nout; ++j) ptrs[nin + j] = p.outputs[j];
  long long n = p.n;
  for (int i = 0; i < nin + nout; ++i) args[i] = &ptrs[i];
  args[nin + nout] = &n;
  static int sm_count[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = dev >= 0 && dev < 64 ? sm_count[dev] : 0;
  if (sms <= 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    if (dev >= 0 && dev < 64) sm_count[dev] = sms;
  }
  const long long groups = n / 4;
  // one two-group iteration per thread where the grid allows (blocks finish
  // together; at 4 blocks an SM and 3-4 iterations a thread, 2^22-element
  // runs took 14.3 us instead of 13.8-14.0), capped at 16 blocks an SM
  const long long blocks = std::max<long long>(1, std::min<long long>((groups + 511) / 512, (long long)sms * 16));
  // launched with programmatic stream serialization (the kernel waits for the
  // previous grid itself); MTL_NO_PDL=1 launches in plain stream order
  static const bool no_pdl = [] {
    const char* v = std::getenv("MTL_NO_PDL");
    return v && v[0] == '1';
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = no_pdl ? 0 : 1;
  cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)kernel, args);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "compiled fused run: %s", cudaGetErrorString(e));
  return MTL_OK;
}

}  // namespace mtl
