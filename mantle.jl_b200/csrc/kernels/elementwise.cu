// Elementwise kernels: every elementwise dispatch — one reference kernel or a
// fused chain of them — runs as a small micro-op program over per-thread
// registers. The program is identical for every thread, so the interpreter's
// branches are warp-uniform; the register file is indexed only by constants
// inside switch cases, so it lives in registers, not local memory.
//
// Loads and stores are 128-bit (float4) and coalesced whenever every pointer is
// 16-byte aligned; each thread handles two float4 per iteration of a grid-stride
// loop sized to a multiple of the SM count.
//
// Floating-point order: every add/sub/mul is an explicit round-to-nearest
// intrinsic, so nothing is contracted into an FMA unless the kernel itself is an
// fma. Results therefore match a CPU that evaluates the same expression in the
// same order bit for bit (sqrt is correctly rounded too); only `sin` may differ
// in the last places.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "../mtl_internal.hpp"

namespace mtl {

constexpr int EW_MAX_IN = 6;
constexpr int EW_MAX_OUT = 8;
constexpr int EW_MAX_OPS = 40;
constexpr int EW_MAX_REGS = 8;

struct EwParams {
  const float* in[EW_MAX_IN];
  float* out[EW_MAX_OUT];
  int8_t out_reg[EW_MAX_OUT];
  int32_t nin, nout, nops;
  int64_t n;
  EwOp ops[EW_MAX_OPS];
};

template <int V>
struct Vec {
  float4 x[V];
};

template <int V>
__device__ __forceinline__ Vec<V> get(const Vec<V> (&r)[EW_MAX_REGS], int i) {
  switch (i) {
#define C(k) \
  case k:    \
    return r[k];
    C(0) C(1) C(2) C(3) C(4) C(5) C(6)
#undef C
    default:
      return r[7];
  }
}

template <int V>
__device__ __forceinline__ void set(Vec<V> (&r)[EW_MAX_REGS], int i, const Vec<V>& v) {
  switch (i) {
#define C(k)  \
  case k:     \
    r[k] = v; \
    break;
    C(0) C(1) C(2) C(3) C(4) C(5) C(6)
#undef C
    default:
      r[7] = v;
  }
}

__device__ __forceinline__ float apply(uint8_t op, float a, float b, float c, float imm) {
  switch (op) {
    case EW_MOV: return a;
    case EW_ADD: return __fadd_rn(a, b);
    case EW_SUB: return __fsub_rn(a, b);
    case EW_MUL: return __fmul_rn(a, b);
    case EW_FMA: return __fmaf_rn(a, b, c);
    case EW_ABS: return fabsf(a);
    case EW_SQRT: return __fsqrt_rn(a);
    case EW_SIN: return sinf(a);
    case EW_MULK: return __fmul_rn(a, imm);
    case EW_ADDK: return __fadd_rn(a, imm);
    default: return imm;
  }
}

template <int V>
__device__ __forceinline__ Vec<V> apply_vec(const EwOp& o, const Vec<V>& a, const Vec<V>& b,
                                            const Vec<V>& c) {
  Vec<V> v;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    v.x[k].x = apply(o.op, a.x[k].x, b.x[k].x, c.x[k].x, o.imm);
    v.x[k].y = apply(o.op, a.x[k].y, b.x[k].y, c.x[k].y, o.imm);
    v.x[k].z = apply(o.op, a.x[k].z, b.x[k].z, c.x[k].z, o.imm);
    v.x[k].w = apply(o.op, a.x[k].w, b.x[k].w, c.x[k].w, o.imm);
  }
  return v;
}

template <int V>
__device__ __forceinline__ void run_program(const EwParams& p, Vec<V> (&r)[EW_MAX_REGS]) {
  for (int k = 0; k < p.nops; ++k) {
    const EwOp o = p.ops[k];
    Vec<V> a = get(r, o.a), b = get(r, o.b), c = get(r, o.c);
    set(r, o.dst, apply_vec(o, a, b, c));
  }
}

// Vectorised body: one float4 per input per thread per iteration, with the
// next iteration's loads issued before this iteration's arithmetic so that two
// groups of loads are in flight per thread.
__global__ void __launch_bounds__(256, 2) ew_vec_kernel(const __grid_constant__ EwParams p) {
  const int64_t groups = p.n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float4 pre[EW_MAX_IN];
#pragma unroll
  for (int i = 0; i < EW_MAX_IN; ++i)
    if (i < p.nin && g < groups) pre[i] = __ldg(reinterpret_cast<const float4*>(p.in[i]) + g);
  for (; g < groups; g += stride) {
    Vec<1> r[EW_MAX_REGS];
#pragma unroll
    for (int i = 0; i < EW_MAX_IN; ++i)
      if (i < p.nin) r[i].x[0] = pre[i];
    const int64_t nx = g + stride;
#pragma unroll
    for (int i = 0; i < EW_MAX_IN; ++i)
      if (i < p.nin && nx < groups) pre[i] = __ldg(reinterpret_cast<const float4*>(p.in[i]) + nx);
    run_program(p, r);
    for (int j = 0; j < p.nout; ++j)
      reinterpret_cast<float4*>(p.out[j])[g] = get(r, p.out_reg[j]).x[0];
  }
  // The ragged tail (at most three elements) is done by the first threads of
  // block 0, one element each, so a launch is always a single kernel.
  const int64_t t = groups * 4 + threadIdx.x;
  if (blockIdx.x == 0 && t < p.n) {
    Vec<1> r[EW_MAX_REGS];
    for (int k = 0; k < p.nin; ++k) {
      Vec<1> v;
      v.x[0].x = v.x[0].y = v.x[0].z = v.x[0].w = p.in[k][t];
      set(r, k, v);
    }
    run_program(p, r);
    for (int j = 0; j < p.nout; ++j) p.out[j][t] = get(r, p.out_reg[j]).x[0].x;
  }
}

// Scalar body, for programs where some pointer is not 16-byte aligned. Uses
// lane 0 of a width-1 vector.
__global__ void __launch_bounds__(256) ew_scalar_kernel(const __grid_constant__ EwParams p,
                                                        int64_t begin) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += stride) {
    Vec<1> r[EW_MAX_REGS];
    for (int k = 0; k < p.nin; ++k) {
      Vec<1> v;
      v.x[0].x = v.x[0].y = v.x[0].z = v.x[0].w = p.in[k][i];
      set(r, k, v);
    }
    run_program(p, r);
    for (int j = 0; j < p.nout; ++j) p.out[j][i] = get(r, p.out_reg[j]).x[0].x;
  }
}

static int sm_count_of_current() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

bool ew_program_fits(const EwProgram& p) {
  return (int)p.inputs.size() <= EW_MAX_IN && (int)p.outputs.size() <= EW_MAX_OUT &&
         (int)p.ops.size() <= EW_MAX_OPS && p.nregs <= EW_MAX_REGS;
}

mtl_status ew_launch_program(const EwProgram& prog, void* stream) {
  if ((int)prog.inputs.size() > EW_MAX_IN || (int)prog.outputs.size() > EW_MAX_OUT ||
      (int)prog.ops.size() > EW_MAX_OPS || prog.nregs > EW_MAX_REGS)
    return fail(MTL_ERR_UNSUPPORTED, "elementwise program too large (%zu in, %zu out, %zu ops, %d regs)",
                prog.inputs.size(), prog.outputs.size(), prog.ops.size(), prog.nregs);
  if (prog.n <= 0 || prog.outputs.empty()) return MTL_OK;
  EwParams p;
  memset(&p, 0, sizeof p);
  p.nin = (int)prog.inputs.size();
  p.nout = (int)prog.outputs.size();
  p.nops = (int)prog.ops.size();
  p.n = prog.n;
  bool aligned = true;
  for (int i = 0; i < p.nin; ++i) {
    p.in[i] = reinterpret_cast<const float*>(prog.inputs[i]);
    aligned &= (prog.inputs[i] % 16) == 0;
  }
  for (int j = 0; j < p.nout; ++j) {
    p.out[j] = reinterpret_cast<float*>(prog.outputs[j]);
    p.out_reg[j] = (int8_t)prog.out_regs[j];
    aligned &= (prog.outputs[j] % 16) == 0;
  }
  for (int k = 0; k < p.nops; ++k) p.ops[k] = prog.ops[k];
  cudaStream_t s = (cudaStream_t)stream;
  const int block = 256;
  const int sms = sm_count_of_current();
  if (aligned) {
    // Two resident blocks per SM; a grid-stride loop covers the rest.
    const int64_t groups = p.n / 4;
    int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((groups + block - 1) / block, (int64_t)sms * 2));
    ew_vec_kernel<<<(unsigned)blocks, block, 0, s>>>(p);
  } else {
    int64_t blocks = std::min<int64_t>((p.n + block - 1) / block, (int64_t)sms * 8);
    ew_scalar_kernel<<<(unsigned)blocks, block, 0, s>>>(p, 0);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "elementwise launch: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// ── the elementwise kernel families ─────────────────────────────────────────
// Each one states, in micro-ops, exactly the expression of the reference kernel
// it stands in for. Registers are SSA values here; `ew_emit` callers compact
// them afterwards.
struct Emitter {
  std::vector<EwOp>& prog;
  int* nregs;
  int op(uint8_t code, int a, int b = 0, int c = 0, float imm = 0.f) {
    int d = (*nregs)++;
    prog.push_back(EwOp{code, (uint8_t)d, (uint8_t)a, (uint8_t)b, (uint8_t)c, imm});
    return d;
  }
};

// Argument access for a kernel's emit: the register of argument i's current
// value (its slot), or a fresh load request.
#define EMIT_FN(name) \
  static int name(const LaunchArgs& la, std::vector<EwOp>& prog, int* slot, int* out, int* nregs)

// stir!(dst, src, k): dst = src*k + sin(src)            bench/independent.jl:37-40
EMIT_FN(emit_stir) {
  Emitter e{prog, nregs};
  int s = slot[1];
  int t = e.op(EW_MULK, s, 0, 0, la.a[2].f32);
  int u = e.op(EW_SIN, s);
  out[0] = e.op(EW_ADD, t, u);
  return 0;
}
// mix!(dst, a, b, k): dst = a*0.5 + b*0.25 + k         bench/fuzz.jl:19-22
EMIT_FN(emit_mix) {
  Emitter e{prog, nregs};
  int t = e.op(EW_MULK, slot[1], 0, 0, 0.5f);
  int u = e.op(EW_MULK, slot[2], 0, 0, 0.25f);
  int v = e.op(EW_ADD, t, u);
  out[0] = e.op(EW_ADDK, v, 0, 0, la.a[3].f32);
  return 0;
}
// keep!(dst, src): dst = src                            bench/fuzz.jl:24-27
EMIT_FN(emit_keep) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_MOV, slot[1]);
  return 0;
}
// touchN!(a, b…): a = a*1.0001 + b + c + d              bench/stress.jl:30-45
static int emit_touch_n(const LaunchArgs&, std::vector<EwOp>& prog, int* slot, int* out, int* nregs,
                        int nsrc) {
  Emitter e{prog, nregs};
  int v = e.op(EW_MULK, slot[0], 0, 0, 1.0001f);
  if (nsrc == 0) {
    v = e.op(EW_ADDK, v, 0, 0, 1.0f);
  } else {
    for (int k = 1; k <= nsrc; ++k) v = e.op(EW_ADD, v, slot[k]);
  }
  out[0] = v;
  return 0;
}
EMIT_FN(emit_touch1) { return emit_touch_n(la, prog, slot, out, nregs, 0); }
EMIT_FN(emit_touch2) { return emit_touch_n(la, prog, slot, out, nregs, 1); }
EMIT_FN(emit_touch3) { return emit_touch_n(la, prog, slot, out, nregs, 2); }
EMIT_FN(emit_touch4) { return emit_touch_n(la, prog, slot, out, nregs, 3); }
// bump!(dst, src, k): dst = src + k                     test/test_window.jl:37-40
EMIT_FN(emit_bump) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_ADDK, slot[1], 0, 0, la.a[2].f32);
  return 0;
}
// scaleby!(dst, src, a): dst = src*a                    test/test_window.jl:84-86
EMIT_FN(emit_scaleby) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_MULK, slot[1], 0, 0, la.a[2].f32);
  return 0;
}
// sched_write!(dst, v): dst = v                         test/test_window.jl:727-730
EMIT_FN(emit_sched_write) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_CONST, 0, 0, 0, la.a[1].f32);
  return 0;
}
// sched_accum!(dst, src): dst += src                    test/test_window.jl:731-734
EMIT_FN(emit_sched_accum) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_ADD, slot[0], slot[1]);
  return 0;
}
// The eight-op chain of the elementwise-chain workload, one op per kernel:
// axpy (a*x + y), mul, add, fma, abs, sqrt(|x|), scale, sub.
EMIT_FN(emit_axpy) {
  Emitter e{prog, nregs};
  int t = e.op(EW_MULK, slot[1], 0, 0, la.a[3].f32);
  out[0] = e.op(EW_ADD, t, slot[2]);
  return 0;
}
EMIT_FN(emit_mul) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_MUL, slot[1], slot[2]);
  return 0;
}
EMIT_FN(emit_add) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_ADD, slot[1], slot[2]);
  return 0;
}
EMIT_FN(emit_sub) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_SUB, slot[1], slot[2]);
  return 0;
}
EMIT_FN(emit_fma) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_FMA, slot[1], slot[2], slot[3]);
  return 0;
}
EMIT_FN(emit_abs) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_ABS, slot[1]);
  return 0;
}
EMIT_FN(emit_sqrt_abs) {
  Emitter e{prog, nregs};
  int t = e.op(EW_ABS, slot[1]);
  out[0] = e.op(EW_SQRT, t);
  return 0;
}
EMIT_FN(emit_scale) {
  Emitter e{prog, nregs};
  out[0] = e.op(EW_MULK, slot[1], 0, 0, la.a[2].f32);
  return 0;
}
// The whole chain in one dispatch: out = 2*sqrt(|fma(0.5x+y)*z+y, x, z)|) - x.
EMIT_FN(emit_chain) {
  Emitter e{prog, nregs};
  int x = slot[1], y = slot[2], z = slot[3];
  int t1 = e.op(EW_ADD, e.op(EW_MULK, x, 0, 0, 0.5f), y);
  int t2 = e.op(EW_MUL, t1, z);
  int t3 = e.op(EW_ADD, t2, y);
  int t4 = e.op(EW_FMA, t3, x, z);
  int t5 = e.op(EW_ABS, t4);
  int t6 = e.op(EW_SQRT, e.op(EW_ABS, t5));
  int t7 = e.op(EW_MULK, t6, 0, 0, 2.0f);
  out[0] = e.op(EW_SUB, t7, x);
  return 0;
}
#undef EMIT_FN

static int arity(uint8_t op) {
  switch (op) {
    case EW_CONST: return 0;
    case EW_ADD: case EW_SUB: case EW_MUL: return 2;
    case EW_FMA: return 3;
    default: return 1;
  }
}

// Compact SSA registers to at most EW_MAX_REGS physical ones (linear scan).
// Operands are read before the destination is written, so an operand whose
// last use is this op gives its register to the result.
static mtl_status compact_registers(EwProgram& p, int nssa) {
  const int nin = (int)p.inputs.size();
  if (nin > EW_MAX_REGS) return fail(MTL_ERR_UNSUPPORTED, "too many elementwise inputs");
  const int END = (int)p.ops.size();
  std::vector<int> last_use(nssa, -1);
  for (int k = 0; k < END; ++k) {
    const EwOp& o = p.ops[k];
    const int ar = arity(o.op);
    const uint8_t src[3] = {o.a, o.b, o.c};
    for (int q = 0; q < ar; ++q) last_use[src[q]] = std::max(last_use[src[q]], k);
  }
  for (int r : p.out_regs) last_use[r] = END;
  std::vector<int> phys(nssa, -1);
  std::vector<int> free_regs;
  for (int r = EW_MAX_REGS - 1; r >= nin; --r) free_regs.push_back(r);
  for (int i = 0; i < nin; ++i) {
    phys[i] = i;
    if (last_use[i] < 0) free_regs.push_back(i);
  }
  for (int k = 0; k < END; ++k) {
    EwOp& o = p.ops[k];
    const int ar = arity(o.op);
    int src[3] = {o.a, o.b, o.c};
    int ph[3] = {0, 0, 0};
    for (int q = 0; q < ar; ++q) ph[q] = phys[src[q]];
    for (int q = 0; q < ar; ++q) {
      bool dup = false;
      for (int r = 0; r < q; ++r) dup |= src[r] == src[q];
      if (!dup && last_use[src[q]] == k) free_regs.push_back(phys[src[q]]);
    }
    if (free_regs.empty())
      return fail(MTL_ERR_UNSUPPORTED, "elementwise program needs more than %d registers", EW_MAX_REGS);
    int d = free_regs.back();
    free_regs.pop_back();
    int dssa = o.dst;
    phys[dssa] = d;
    if (last_use[dssa] < 0) free_regs.push_back(d);  // dead result
    o.a = (uint8_t)ph[0];
    o.b = (uint8_t)ph[1];
    o.c = (uint8_t)ph[2];
    o.dst = (uint8_t)d;
  }
  for (int& r : p.out_regs) r = phys[r];
  int maxr = nin;
  for (auto& o : p.ops) maxr = std::max(maxr, (int)o.dst + 1);
  p.nregs = maxr;
  return MTL_OK;
}

}  // namespace mtl

// Builds the program for a sequence of elementwise dispatches (one, or a fused
// chain). A buffer read before the chain writes it is loaded once at the start;
// every written buffer is stored once at the end, except the keys in `elided`
// (graph resources with rid r appear as (1<<63)|r): intermediates nothing
// outside the chain reads.
namespace mtl {
mtl_status ew_build_program(const std::vector<EwMember>& ms, const std::vector<uint64_t>& elided,
                            EwProgram& out) {
  out = EwProgram();
  // Buffers are keyed by graph resource when they have one (elided transients
  // have no address), else by pointer.
  auto key = [](const Arg& a) -> uint64_t { return a.rid ? ((uint64_t)1 << 63) | (uint64_t)a.rid : a.ptr; };
  std::map<uint64_t, int> reg_of;      // buffer -> SSA register with its current value
  std::map<uint64_t, uint64_t> ptr_of; // buffer key -> device pointer
  std::vector<uint64_t> written_order; // buffers written, first-write order
  std::vector<EwOp> ops;
  int nssa = 0;
  // Pass 1: discover the inputs (buffers read before being written in the chain).
  std::vector<uint64_t> in_keys;
  {
    std::set<uint64_t> defined;
    for (const EwMember& m : ms) {
      for (size_t i = 0; i < m.la.a.size(); ++i) {
        if (!(m.kd->reads_mask >> i & 1)) continue;
        uint64_t k = key(m.la.a[i]);
        ptr_of[k] = m.la.a[i].ptr;
        if (!defined.count(k) && std::find(in_keys.begin(), in_keys.end(), k) == in_keys.end()) {
          in_keys.push_back(k);
          out.inputs.push_back(m.la.a[i].ptr);
        }
      }
      for (size_t i = 0; i < m.la.a.size(); ++i)
        if (m.kd->writes_mask >> i & 1) {
          defined.insert(key(m.la.a[i]));
          ptr_of[key(m.la.a[i])] = m.la.a[i].ptr;
        }
    }
  }
  nssa = (int)in_keys.size();
  for (int i = 0; i < (int)in_keys.size(); ++i) reg_of[in_keys[i]] = i;
  int64_t n = -1;
  for (const EwMember& m : ms) {
    if (n < 0) n = m.la.nd[0];
    if (m.la.nd[0] != n) return fail(MTL_ERR_ARGUMENT, "fused elementwise dispatches disagree on ndrange");
    int slot[16], outr[16];
    for (int i = 0; i < 16; ++i) slot[i] = outr[i] = -1;
    for (size_t i = 0; i < m.la.a.size() && i < 16; ++i) {
      if (m.la.a[i].kind != MTL_ARG_PTR) continue;
      auto it = reg_of.find(key(m.la.a[i]));
      if (it != reg_of.end()) slot[i] = it->second;
    }
    for (size_t i = 0; i < m.la.a.size(); ++i)
      if ((m.kd->reads_mask >> i & 1) && slot[i] < 0)
        return fail(MTL_ERR_ARGUMENT, "elementwise argument %zu read before it has a value", i + 1);
    m.kd->ew_emit(m.la, ops, slot, outr, &nssa);
    // emit_* write out[0] for the (single) written argument; map it.
    int wi = 0;
    for (size_t i = 0; i < m.la.a.size(); ++i)
      if (m.kd->writes_mask >> i & 1) {
        uint64_t k = key(m.la.a[i]);
        reg_of[k] = outr[wi++];
        if (std::find(written_order.begin(), written_order.end(), k) == written_order.end())
          written_order.push_back(k);
      }
  }
  for (uint64_t k : written_order) {
    if (std::find(elided.begin(), elided.end(), k) != elided.end()) continue;
    out.outputs.push_back(ptr_of[k]);
    out.out_regs.push_back(reg_of[k]);
  }
  out.ops = ops;
  out.n = n < 0 ? 0 : n;
  return compact_registers(out, nssa);
}

// Launch one elementwise dispatch on its own.
mtl_status ew_launch_single(const KernelDesc* kd, const LaunchArgs& la, void* stream) {
  std::vector<EwMember> ms = {EwMember{kd, la}};
  EwProgram p;
  mtl_status st = ew_build_program(ms, {}, p);
  if (st) return st;
  return ew_launch_program(p, stream);
}

// Emit-function table, consumed by the kernel registry.
int (*ew_emit_fn(const char* name))(const LaunchArgs&, std::vector<EwOp>&, int*, int*, int*) {
  struct E {
    const char* n;
    int (*f)(const LaunchArgs&, std::vector<EwOp>&, int*, int*, int*);
  };
  static const E table[] = {
      {"stir", emit_stir},        {"mix", emit_mix},         {"keep", emit_keep},
      {"touch1", emit_touch1},    {"touch2", emit_touch2},   {"touch3", emit_touch3},
      {"touch4", emit_touch4},    {"bump", emit_bump},       {"scaleby", emit_scaleby},
      {"sched_write", emit_sched_write}, {"sched_accum", emit_sched_accum},
      {"axpy", emit_axpy},        {"mul", emit_mul},         {"add", emit_add},
      {"sub", emit_sub},          {"fma", emit_fma},         {"abs", emit_abs},
      {"sqrt_abs", emit_sqrt_abs}, {"scale", emit_scale},    {"chain8", emit_chain},
  };
  for (const E& e : table)
    if (!strcmp(e.n, name)) return e.f;
  return nullptr;
}

}  // namespace mtl
