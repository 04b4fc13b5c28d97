// The CUDA side of the backend: devices, persistent buffers, and plans — a
// compiled Mantle graph lowered to one CUDA graph and replayed with a single
// cudaGraphLaunch per run! (a plan that is one kernel, with no updates and no
// profiling, launches that kernel directly instead).
//
// Lowering (ext/MantleLavaExt.jl:2076-2338 is what it replaces):
//   * every dispatch becomes a child-graph node captured from its launch(es),
//     so a kernel that needs two launches (scatter + reduce) is still one node;
//   * a custom! body is captured the same way, once per instantiation;
//   * the shared update pass becomes memcpy nodes (pinned staging or device
//     source), enabled only on frames that have pending data;
//   * copy! becomes a device-to-device memcpy node;
//   * the derived hazards become the node dependencies; :backend chains every
//     pass (and every dispatch) in scheduled order, as an unconditional barrier
//     after each dispatch would;
//   * profile = true brackets every pass with event-record nodes.
// Launches of one exec graph on one stream run in order, so frame N+1 never
// overlaps frame N and no cross-frame edge is needed.

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <deque>
#include <functional>

#include "mtl_internal.hpp"

using namespace mtl;

struct mtl_device {
  std::atomic<int> refs{1};  // the handle + every graph, buffer and communicator on it
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  int sm_count = 148;
  int64_t l2 = 0, hbm = 0;
  int cc_major = 0, cc_minor = 0;
  uint64_t pool_cap = 0;   // 0 = none
  uint64_t pool_used = 0;  // bytes of live plan slabs
};

struct mtl_buffer {
  std::atomic<int> refs{1};  // the handle + every graph that names it
  mtl_device* dev = nullptr;
  void* ptr = nullptr;
  uint64_t bytes = 0;
  bool owned = true;
};

namespace mtl {
int device_sm_count(mtl_device* d) { return d ? d->sm_count : 148; }

void retain_device(mtl_device* d) { d->refs.fetch_add(1); }
void release_device(mtl_device* d) {
  if (d->refs.fetch_sub(1) != 1) return;
  cudaSetDevice(d->ordinal);
  if (d->stream) {
    cudaStreamSynchronize(d->stream);
    cudaStreamDestroy(d->stream);
  }
  delete d;
}
void retain_buffer(mtl_buffer* b) { b->refs.fetch_add(1); }
void release_buffer(mtl_buffer* b) {
  if (b->refs.fetch_sub(1) != 1) return;
  mtl_device* d = b->dev;
  if (b->owned && b->ptr) {
    if (d) {
      cudaSetDevice(d->ordinal);
      cudaStreamSynchronize(d->stream);
    }
    cudaFree(b->ptr);
  }
  delete b;
  if (d) release_device(d);
}
int device_ordinal(mtl_device* d) { return d ? d->ordinal : -1; }
}

#define CUDA_TRY(expr)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (expr);                                                                 \
    if (e_ != cudaSuccess) return fail(MTL_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

static mtl_status use_device(mtl_device* d) {
  if (!d) return fail(MTL_ERR_STATE, "no device");
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur == d->ordinal) return MTL_OK;
  CUDA_TRY(cudaSetDevice(d->ordinal));
  return MTL_OK;
}

// ── plan ────────────────────────────────────────────────────────────────────
namespace {

constexpr int kStagingSlots = 3;
constexpr size_t kNSamples = 120;  // NSAMPLES, src/runtime/api.jl:246

struct ModeGraph {
  bool built = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // By scheduled position: node of each dispatch (compute passes), and the
  // nodes a dependent has to wait for.
  std::vector<std::vector<cudaGraphNode_t>> dispatch_nodes;
  std::vector<std::vector<cudaGraphNode_t>> exit_nodes;
  std::vector<cudaGraphNode_t> upd_host, upd_dev;
  std::vector<int8_t> upd_host_on, upd_dev_on;
  int nkernels = 0, nedges = 0;
  std::function<mtl_status(cudaStream_t)> direct;  // set for one-kernel plans (direct_launcher)
};

struct UpdateRt {
  uint64_t dst = 0;         // device address written
  uint64_t max_bytes = 0;   // declared range, or the whole buffer
  void* staging[kStagingSlots] = {};
  cudaEvent_t ev[kStagingSlots] = {};
  bool ev_used[kStagingSlots] = {};
  int next = 0;
  const void* pending = nullptr;
  uint64_t pending_bytes = 0;
  bool pending_dev = false;
  bool pending_pinned = false;  // page-locked host memory: copied by DMA directly
};

}  // namespace

struct mtl_plan {
  mtl_graph* g = nullptr;
  CompileOpts o;
  Analysis a;
  void* slab = nullptr;
  uint64_t slab_bytes = 0;
  ModeGraph modes[2];
  std::vector<UpdateRt> upd;
  cudaStream_t capture = nullptr;
  // profiler
  std::vector<cudaEvent_t> ev_start, ev_end;
  std::vector<std::deque<double>> gpu_ms, host_ms;
  bool prof_pending = false;
  int prof_mode = 0;
};

static uint64_t resource_bytes(const mtl_graph* g, int rid) {
  const Resource& r = g->res[rid - 1];
  if (r.kind == RES_VIEW) return resource_bytes(g, r.parent);
  return r.elems * r.elem_bytes;
}

static uint64_t resource_ptr(const mtl_plan* pl, int rid) {
  const mtl_graph* g = pl->g;
  const Resource& r = g->res[rid - 1];
  switch (r.kind) {
    case RES_PERSISTENT: return r.buf ? (uint64_t)r.buf->ptr : 0;
    case RES_TRANSIENT: return (uint64_t)pl->slab + (uint64_t)pl->a.offsets[r.transient_index];
    default: return resource_ptr(pl, r.parent);  // a slice binds its whole buffer
  }
}

static mtl_status resolve(const mtl_plan* pl, const Dispatch& d, LaunchArgs& la, void** ws,
                          uint64_t* ws_bytes) {
  la.a.clear();
  la.ndim = d.ndim;
  for (int i = 0; i < 3; ++i) {
    la.nd[i] = i < d.ndim ? d.nd[i] : 1;
    la.group[i] = d.group[i];
  }
  la.sm_count = device_sm_count(pl->g->dev);
  la.device = device_ordinal(pl->g->dev);
  for (const mtl_arg& m : d.args) {
    Arg x;
    switch (m.kind) {
      case MTL_ARG_RESOURCE:
        x.kind = MTL_ARG_PTR;
        x.ptr = resource_ptr(pl, m.rid);
        x.bytes = resource_bytes(pl->g, m.rid);
        x.rid = m.rid;
        break;
      case MTL_ARG_PTR:
        x.kind = MTL_ARG_PTR;
        x.ptr = m.v.ptr;
        x.bytes = m.bytes;
        break;
      case MTL_ARG_F32: x.kind = m.kind; x.f32 = m.v.f32; break;
      case MTL_ARG_I32: x.kind = m.kind; x.i32 = m.v.i32; break;
      case MTL_ARG_I64: x.kind = m.kind; x.i64 = m.v.i64; break;
      case MTL_ARG_F64: x.kind = m.kind; x.f64 = m.v.f64; break;
      default: x.kind = MTL_ARG_NULL;
    }
    la.a.push_back(x);
  }
  *ws = nullptr;
  *ws_bytes = 0;
  if (d.workspace_rid) {
    *ws = (void*)resource_ptr(pl, d.workspace_rid);
    *ws_bytes = resource_bytes(pl->g, d.workspace_rid);
  }
  return MTL_OK;
}

static int count_kernels(cudaGraph_t g) {
  size_t n = 0;
  cudaGraphGetNodes(g, nullptr, &n);
  std::vector<cudaGraphNode_t> nodes(n);
  if (n) cudaGraphGetNodes(g, nodes.data(), &n);
  int k = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType t;
    cudaGraphNodeGetType(nd, &t);
    if (t == cudaGraphNodeTypeKernel) ++k;
    if (t == cudaGraphNodeTypeGraph) {
      cudaGraph_t c;
      cudaGraphChildGraphNodeGetGraph(nd, &c);
      k += count_kernels(c);
    }
  }
  return k;
}

// Capture `body` on the plan's capture stream into a child graph.
static mtl_status capture_graph(mtl_plan* pl, const std::function<mtl_status(cudaStream_t)>& body,
                                cudaGraph_t* out) {
  CUDA_TRY(cudaStreamBeginCapture(pl->capture, cudaStreamCaptureModeRelaxed));
  mtl_status st = body(pl->capture);
  std::string msg = st ? mtl_last_error() : "";
  cudaGraph_t child = nullptr;
  cudaError_t e = cudaStreamEndCapture(pl->capture, &child);
  if (st) {
    if (child) cudaGraphDestroy(child);
    return fail(st, "%s", msg.c_str());
  }
  if (e != cudaSuccess) {
    if (child) cudaGraphDestroy(child);
    return fail(MTL_ERR_CUDA, "stream capture: %s", cudaGetErrorString(e));
  }
  *out = child;
  return MTL_OK;
}

using Launcher = std::function<mtl_status(cudaStream_t)>;

// What a dispatch launches, with its resources resolved to this plan's memory.
static Launcher dispatch_launcher(mtl_plan* pl, const Dispatch& d) {
  LaunchArgs la;
  void* ws;
  uint64_t wsb;
  resolve(pl, d, la, &ws, &wsb);
  const int kernel = d.kernel;
  return [kernel, la, ws, wsb](cudaStream_t s) { return launch_kernel(kernel, la, ws, wsb, s); };
}

static mtl_status capture_dispatch(mtl_plan* pl, const Dispatch& d, cudaGraph_t* out) {
  return capture_graph(pl, dispatch_launcher(pl, d), out);
}

// Whether scheduled position p runs as one compiled elementwise program: a
// fused run, or a single elementwise pass (compiled too: the interpreter
// kernel moves ~1.1 TB/s, the compiled kernel of the same op ~5).
static bool compiled_step(const mtl_plan* pl, int p) {
  const auto& st = pl->a.steps[p];
  return st.size() > 1 || (st.size() == 1 && mtl_pass_compilable(pl->g, st[0]));
}

// A fused run of elementwise passes (scheduled position p): one program, one
// kernel. Transients the run keeps in registers are never stored.
static mtl_status fused_launcher(mtl_plan* pl, int p, Launcher* out) {
  const mtl_graph* g = pl->g;
  std::vector<EwMember> ms;
  for (int pid : pl->a.steps[p]) {
    const Dispatch& d = g->passes[pid].dispatches[0];
    EwMember m;
    m.kd = kernel_desc(d.kernel);
    void* ws;
    uint64_t wsb;
    resolve(pl, d, m.la, &ws, &wsb);
    std::vector<uint64_t> bytes(m.la.a.size());
    for (size_t i = 0; i < m.la.a.size(); ++i) bytes[i] = m.la.a[i].bytes;
    if (mtl_status s = m.kd->check(m.la, bytes.data())) return s;
    ms.push_back(m);
  }
  std::vector<uint64_t> elided;
  for (int rid : pl->a.elided) elided.push_back(((uint64_t)1 << 63) | (uint64_t)rid);
  EwProgram prog;
  if (mtl_status s = ew_build_program(ms, elided, prog)) return s;
  // Straight-line code for the run, compiled now (never per frame); the
  // interpreter kernel when that is not possible here.
  bool aligned = prog.n > 0 && ew_program_fits(prog);
  for (uint64_t x : prog.inputs) aligned &= x % 16 == 0;
  for (uint64_t x : prog.outputs) aligned &= x % 16 == 0;
  void* compiled = nullptr;
  if (aligned) {
    mtl_status st = ew_compile(prog, &compiled);
    if (st != MTL_OK && st != MTL_ERR_UNSUPPORTED) return st;  // NVRTC present but failing: an error
  }
  if (compiled)
    *out = [compiled, prog](cudaStream_t s) { return ew_launch_compiled(compiled, prog, s); };
  else
    *out = [prog](cudaStream_t s) { return ew_launch_program(prog, s); };
  return MTL_OK;
}

static mtl_status capture_fused(mtl_plan* pl, int p, cudaGraph_t* out) {
  Launcher f;
  if (mtl_status s = fused_launcher(pl, p, &f)) return s;
  return capture_graph(pl, f, out);
}

// A plan that is one step launching one kernel, with no updates and no
// profiling, runs that launch directly on the device stream: back-to-back
// kernel launches leave shorter gaps on the GPU than launches of one-node
// graphs (measured ~3.5 us between replays of the fused chain's graph).
static mtl_status direct_launcher(mtl_plan* pl, const ModeGraph& m, Launcher* out) {
  *out = nullptr;
  const mtl_graph* g = pl->g;
  if (pl->a.order.size() != 1 || !g->updates.empty() || pl->o.profile || m.nkernels != 1) return MTL_OK;
  if (compiled_step(pl, 0)) return fused_launcher(pl, 0, out);
  const Pass& ps = g->passes[pl->a.order[0]];
  if (ps.kind == MTL_PASS_COMPUTE && ps.dispatches.size() == 1) *out = dispatch_launcher(pl, ps.dispatches[0]);
  return MTL_OK;
}

// Scheduled position of a pass (the step that runs it), or -1.
static int position_of(const mtl_plan* pl, int pass) {
  for (size_t p = 0; p < pl->a.steps.size(); ++p)
    for (int m : pl->a.steps[p])
      if (m == pass) return (int)p;
  return -1;
}

static mtl_status add_child(cudaGraph_t parent, const std::vector<cudaGraphNode_t>& deps,
                            cudaGraph_t child, cudaGraphNode_t* node) {
  CUDA_TRY(cudaGraphAddChildGraphNode(node, parent, deps.data(), deps.size(), child));
  return MTL_OK;
}

static void destroy_mode(ModeGraph& m) {
  if (m.exec) cudaGraphExecDestroy(m.exec);
  if (m.graph) cudaGraphDestroy(m.graph);
  m = ModeGraph();
}

static mtl_status build_mode(mtl_plan* pl, int mode) {
  ModeGraph& m = pl->modes[mode];
  if (m.built) return MTL_OK;
  mtl_graph* g = pl->g;
  const Analysis& a = pl->a;
  const int n = (int)a.order.size();
  CUDA_TRY(cudaGraphCreate(&m.graph, 0));
  m.dispatch_nodes.assign(n, {});
  m.exit_nodes.assign(n, {});
  m.upd_host.assign(g->updates.size(), nullptr);
  m.upd_dev.assign(g->updates.size(), nullptr);
  m.upd_host_on.assign(g->updates.size(), 1);
  m.upd_dev_on.assign(g->updates.size(), 1);
  m.nkernels = 0;
  m.nedges = 0;
  const bool serial = mode == 1;
  for (int p = 0; p < n; ++p) {
    const Pass& ps = g->passes[a.order[p]];
    std::vector<cudaGraphNode_t> entry;
    if (serial) {
      if (p > 0) entry = m.exit_nodes[p - 1];
      m.nedges += p > 0;
    } else {
      for (int q : a.edges[p])
        for (auto nd : m.exit_nodes[q - 1]) entry.push_back(nd);
      m.nedges += (int)a.edges[p].size();
    }
    if (pl->o.profile) {
      cudaGraphNode_t ev;
      CUDA_TRY(cudaGraphAddEventRecordNode(&ev, m.graph, entry.data(), entry.size(), pl->ev_start[p]));
      entry = {ev};
    }
    std::vector<cudaGraphNode_t> body;
    if (compiled_step(pl, p)) {
      cudaGraph_t child = nullptr;
      mtl_status st = capture_fused(pl, p, &child);
      if (st) return fail(st, "fused run from \"%s\": %s", ps.name.c_str(), std::string(mtl_last_error()).c_str());
      m.nkernels += count_kernels(child);
      cudaGraphNode_t nd;
      st = add_child(m.graph, entry, child, &nd);
      cudaGraphDestroy(child);
      if (st) return st;
      m.dispatch_nodes[p].push_back(nd);
      body.push_back(nd);
    } else if (ps.kind == MTL_PASS_COMPUTE) {
      std::vector<cudaGraphNode_t> prev = entry;
      for (const Dispatch& d : ps.dispatches) {
        cudaGraph_t child = nullptr;
        mtl_status st = capture_dispatch(pl, d, &child);
        if (st) return fail(st, "pass \"%s\": %s", ps.name.c_str(), std::string(mtl_last_error()).c_str());
        m.nkernels += count_kernels(child);
        cudaGraphNode_t nd;
        st = add_child(m.graph, serial ? prev : entry, child, &nd);
        cudaGraphDestroy(child);
        if (st) return st;
        m.dispatch_nodes[p].push_back(nd);
        body.push_back(nd);
        if (serial) prev = {nd};
      }
      if (serial && !body.empty()) body = {body.back()};
    } else if (ps.kind == MTL_PASS_CUSTOM) {
      cudaGraph_t child = nullptr;
      mtl_custom_fn fn = ps.custom_fn;
      void* user = ps.custom_user;
      if (!fn) return fail(MTL_ERR_ARGUMENT, "custom! pass \"%s\" has no body", ps.name.c_str());
      mtl_status st = capture_graph(pl, [&](cudaStream_t s) -> mtl_status {
        int32_t r = fn(user, (void*)s, pl);
        if (r != 0) return fail(MTL_ERR_ARGUMENT, "custom! body of \"%s\" returned %d", ps.name.c_str(), r);
        return MTL_OK;
      }, &child);
      if (st) return st;
      m.nkernels += count_kernels(child);
      cudaGraphNode_t nd;
      st = add_child(m.graph, entry, child, &nd);
      cudaGraphDestroy(child);
      if (st) return st;
      body.push_back(nd);
    } else if (ps.kind == MTL_PASS_UPDATE) {
      for (size_t u = 0; u < g->updates.size(); ++u) {
        UpdateRt& ur = pl->upd[u];
        cudaGraphNode_t h, dv;
        CUDA_TRY(cudaGraphAddMemcpyNode1D(&h, m.graph, entry.data(), entry.size(), (void*)ur.dst,
                                          ur.staging[0], ur.max_bytes, cudaMemcpyHostToDevice));
        // The device route's source is patched per frame; at instantiation it
        // names the destination itself, and the node starts disabled.
        CUDA_TRY(cudaGraphAddMemcpyNode1D(&dv, m.graph, entry.data(), entry.size(), (void*)ur.dst,
                                          (void*)ur.dst, ur.max_bytes, cudaMemcpyDeviceToDevice));
        m.upd_host[u] = h;
        m.upd_dev[u] = dv;
        body.push_back(h);
        body.push_back(dv);
      }
    } else if (ps.kind == MTL_PASS_COPY) {
      cudaGraphNode_t nd;
      uint64_t bytes = resource_bytes(g, ps.copy_src);
      CUDA_TRY(cudaGraphAddMemcpyNode1D(&nd, m.graph, entry.data(), entry.size(),
                                        (void*)resource_ptr(pl, ps.copy_dst),
                                        (void*)resource_ptr(pl, ps.copy_src), bytes,
                                        cudaMemcpyDeviceToDevice));
      body.push_back(nd);
    }
    if (body.empty()) {
      cudaGraphNode_t nd;
      CUDA_TRY(cudaGraphAddEmptyNode(&nd, m.graph, entry.data(), entry.size()));
      body.push_back(nd);
    }
    if (pl->o.profile) {
      cudaGraphNode_t ev;
      CUDA_TRY(cudaGraphAddEventRecordNode(&ev, m.graph, body.data(), body.size(), pl->ev_end[p]));
      body = {ev};
    }
    m.exit_nodes[p] = body;
  }
  CUDA_TRY(cudaGraphInstantiate(&m.exec, m.graph, 0));
  for (size_t u = 0; u < g->updates.size(); ++u) {
    CUDA_TRY(cudaGraphNodeSetEnabled(m.exec, m.upd_host[u], 0));
    CUDA_TRY(cudaGraphNodeSetEnabled(m.exec, m.upd_dev[u], 0));
    m.upd_host_on[u] = m.upd_dev_on[u] = 0;
  }
  if (mtl_status st = direct_launcher(pl, m, &m.direct)) return st;
  m.built = true;
  return MTL_OK;
}

static void plan_free(mtl_plan* pl) {
  if (!pl) return;
  if (pl->g && pl->g->dev) {
    cudaSetDevice(pl->g->dev->ordinal);
    if (pl->g->dev->stream) cudaStreamSynchronize(pl->g->dev->stream);
    for (auto& m : pl->modes) destroy_mode(m);
    for (auto& u : pl->upd)
      for (int k = 0; k < kStagingSlots; ++k) {
        if (u.staging[k]) cudaFreeHost(u.staging[k]);
        if (u.ev[k]) cudaEventDestroy(u.ev[k]);
      }
    for (auto e : pl->ev_start) cudaEventDestroy(e);
    for (auto e : pl->ev_end) cudaEventDestroy(e);
    if (pl->slab) {
      cudaFreeAsync(pl->slab, pl->g->dev->stream);
      cudaStreamSynchronize(pl->g->dev->stream);
      pl->g->dev->pool_used -= pl->slab_bytes;
    }
    if (pl->capture) cudaStreamDestroy(pl->capture);
  }
  mtl_graph* g = pl->g;
  delete pl;
  if (g) release_graph(g);
}

static double median(std::deque<double> v) {
  if (v.empty()) return NAN;
  std::sort(v.begin(), v.end());
  return v[v.size() / 2];
}

static void sample(std::deque<double>& ring, double x) {
  ring.push_back(x);
  while (ring.size() > kNSamples) ring.pop_front();
}

// Read the last profiled frame's events without waiting (collect!,
// ext/MantleLavaExt.jl:1986-2006): a frame still in flight is skipped.
static void collect(mtl_plan* pl) {
  if (!pl->o.profile || !pl->prof_pending) return;
  const int n = (int)pl->a.order.size();
  if (n > 0 && cudaEventQuery(pl->ev_end[n - 1]) != cudaSuccess) {
    // Not back yet; check every pass's end event before giving up.
    bool all = true;
    for (int p = 0; p < n && all; ++p) all = cudaEventQuery(pl->ev_end[p]) == cudaSuccess;
    if (!all) {
      cudaGetLastError();
      pl->prof_pending = false;
      return;
    }
  }
  for (int p = 0; p < n; ++p) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, pl->ev_start[p], pl->ev_end[p]) == cudaSuccess && ms >= 0)
      sample(pl->gpu_ms[p], ms);
  }
  cudaGetLastError();
  pl->prof_pending = false;
}

extern "C" {

// ── device ──────────────────────────────────────────────────────────────────
mtl_status mtl_device_open(int32_t ordinal, uint64_t pool_cap_bytes, mtl_device** out) {
  if (!out) return fail(MTL_ERR_ARGUMENT, "mtl_device_open: out is NULL");
  if (mtl_status s = injected("mtl_device_open")) return s;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(MTL_ERR_STATE, "no CUDA device available (%s)", cudaGetErrorString(e));
  if (ordinal < 0 || ordinal >= count)
    return fail(MTL_ERR_ARGUMENT, "device %d does not exist (%d visible)", ordinal, count);
  CUDA_TRY(cudaSetDevice(ordinal));
  auto* d = new mtl_device();
  d->ordinal = ordinal;
  d->pool_cap = pool_cap_bytes;
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, ordinal));
  d->sm_count = prop.multiProcessorCount;
  d->l2 = prop.l2CacheSize;
  d->hbm = (int64_t)prop.totalGlobalMem;
  d->cc_major = prop.major;
  d->cc_minor = prop.minor;
  e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete d;
    return fail(MTL_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
  }
  // Keep freed plan slabs in the pool: plans are rebuilt with the same sizes.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  *out = d;
  return MTL_OK;
}

mtl_status mtl_device_close(mtl_device* d) {
  if (d) release_device(d);
  return MTL_OK;
}

mtl_status mtl_device_synchronize(mtl_device* d) {
  if (mtl_status s = use_device(d)) return s;
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  return MTL_OK;
}

mtl_status mtl_device_stream(mtl_device* d, void** stream) {
  if (!d || !stream) return fail(MTL_ERR_ARGUMENT, "mtl_device_stream: NULL argument");
  *stream = (void*)d->stream;
  return MTL_OK;
}

mtl_status mtl_device_info(mtl_device* d, int32_t* sm_count, int64_t* l2_bytes, int64_t* hbm_bytes,
                           int32_t* cc_major, int32_t* cc_minor) {
  if (!d) return fail(MTL_ERR_ARGUMENT, "no device");
  if (sm_count) *sm_count = d->sm_count;
  if (l2_bytes) *l2_bytes = d->l2;
  if (hbm_bytes) *hbm_bytes = d->hbm;
  if (cc_major) *cc_major = d->cc_major;
  if (cc_minor) *cc_minor = d->cc_minor;
  return MTL_OK;
}

// ── buffers ─────────────────────────────────────────────────────────────────
mtl_status mtl_buffer_alloc(mtl_device* d, uint64_t bytes, mtl_buffer** out) {
  if (!out) return fail(MTL_ERR_ARGUMENT, "mtl_buffer_alloc: out is NULL");
  if (mtl_status s = injected("mtl_buffer_alloc")) return s;
  if (mtl_status s = use_device(d)) return s;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, std::max<uint64_t>(bytes, 1));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MTL_ERR_OOM, "cudaMalloc(%llu): %s", (unsigned long long)bytes, cudaGetErrorString(e));
  }
  auto* b = new mtl_buffer();
  b->dev = d;
  b->ptr = p;
  b->bytes = bytes;
  retain_device(d);
  *out = b;
  return MTL_OK;
}

mtl_status mtl_buffer_wrap(mtl_device* d, void* ptr, uint64_t bytes, mtl_buffer** out) {
  if (!out || !ptr) return fail(MTL_ERR_ARGUMENT, "mtl_buffer_wrap: NULL argument");
  auto* b = new mtl_buffer();
  b->dev = d;
  b->ptr = ptr;
  b->bytes = bytes;
  b->owned = false;
  if (d) retain_device(d);
  *out = b;
  return MTL_OK;
}

mtl_status mtl_buffer_upload(mtl_buffer* b, const void* host, uint64_t off, uint64_t bytes) {
  if (!b || (!host && bytes)) return fail(MTL_ERR_ARGUMENT, "mtl_buffer_upload: NULL argument");
  if (off + bytes > b->bytes)
    return fail(MTL_ERR_ARGUMENT, "update!: bytes %llu..%llu are outside the %llu-byte buffer",
                (unsigned long long)off, (unsigned long long)(off + bytes), (unsigned long long)b->bytes);
  if (mtl_status s = use_device(b->dev)) return s;
  if (!bytes) return MTL_OK;
  CUDA_TRY(cudaMemcpyAsync((char*)b->ptr + off, host, bytes, cudaMemcpyDefault, b->dev->stream));
  CUDA_TRY(cudaStreamSynchronize(b->dev->stream));
  return MTL_OK;
}

mtl_status mtl_buffer_download(mtl_buffer* b, void* host, uint64_t off, uint64_t bytes) {
  if (!b || (!host && bytes)) return fail(MTL_ERR_ARGUMENT, "mtl_buffer_download: NULL argument");
  if (off + bytes > b->bytes)
    return fail(MTL_ERR_ARGUMENT, "Array: bytes %llu..%llu are outside the %llu-byte buffer",
                (unsigned long long)off, (unsigned long long)(off + bytes), (unsigned long long)b->bytes);
  if (mtl_status s = use_device(b->dev)) return s;
  if (!bytes) return MTL_OK;
  CUDA_TRY(cudaMemcpyAsync(host, (char*)b->ptr + off, bytes, cudaMemcpyDefault, b->dev->stream));
  CUDA_TRY(cudaStreamSynchronize(b->dev->stream));
  return MTL_OK;
}

mtl_status mtl_buffer_device_ptr(mtl_buffer* b, void** p) {
  if (!b || !p) return fail(MTL_ERR_ARGUMENT, "mtl_buffer_device_ptr: NULL argument");
  *p = b->ptr;
  return MTL_OK;
}

mtl_status mtl_buffer_release(mtl_buffer* b) {
  if (b) release_buffer(b);
  return MTL_OK;
}

// ── plans ───────────────────────────────────────────────────────────────────
mtl_status mtl_plan_compile(mtl_graph* g, const mtl_plan_opts* opts, mtl_plan** out) {
  if (!g || !out) return fail(MTL_ERR_ARGUMENT, "Plan: NULL argument");
  if (mtl_status s = injected("mtl_plan_compile")) return s;
  auto* pl = new mtl_plan();
  pl->g = g;
  retain_graph(g);  // the plan keeps its graph (and through it the buffers) alive
  if (opts) {
    pl->o.coalesce = opts->coalesce != 0;
    pl->o.alias = opts->alias != 0;
    pl->o.profile = opts->profile != 0;
    pl->o.policy = opts->policy;
    pl->o.fuse = opts->fuse != 0;
  }
  if (pl->o.policy != MTL_POLICY_OVERLAP && pl->o.policy != MTL_POLICY_COMPACT) {
    plan_free(pl);
    return fail(MTL_ERR_ARGUMENT, "Plan: unknown policy %d", pl->o.policy);
  }
  mtl_status st = analyze(g, pl->o, pl->a);
  if (st) {
    plan_free(pl);
    return st;
  }
  if (!g->dev) {  // analysis only
    *out = pl;
    return MTL_OK;
  }
  mtl_device* d = g->dev;
  if ((st = use_device(d))) {
    plan_free(pl);
    return st;
  }
  // Every persistent resource named by the graph must have storage.
  for (size_t i = 0; i < g->res.size(); ++i)
    if (g->res[i].kind == RES_PERSISTENT && !g->res[i].buf) {
      plan_free(pl);
      return fail(MTL_ERR_ARGUMENT, "Plan: resource %zu has no buffer", i + 1);
    }
  auto cleanup = [&](mtl_status s) {
    std::string msg = mtl_last_error();
    plan_free(pl);
    return fail(s, "%s", msg.c_str());
  };
  pl->slab_bytes = (uint64_t)pl->a.peak;
  if (pl->slab_bytes) {
    if (d->pool_cap && d->pool_used + pl->slab_bytes > d->pool_cap) {
      fail(MTL_ERR_OOM, "Plan: the transient slab needs %llu bytes and the pool cap leaves %llu",
           (unsigned long long)pl->slab_bytes, (unsigned long long)(d->pool_cap - d->pool_used));
      return cleanup(MTL_ERR_OOM);
    }
    cudaError_t e = cudaMallocAsync(&pl->slab, pl->slab_bytes, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) {
      cudaGetLastError();
      pl->slab = nullptr;
      fail(MTL_ERR_OOM, "Plan: slab of %llu bytes: %s", (unsigned long long)pl->slab_bytes, cudaGetErrorString(e));
      return cleanup(MTL_ERR_OOM);
    }
    d->pool_used += pl->slab_bytes;
  }
  if (cudaStreamCreateWithFlags(&pl->capture, cudaStreamNonBlocking) != cudaSuccess) {
    fail(MTL_ERR_CUDA, "Plan: capture stream");
    return cleanup(MTL_ERR_CUDA);
  }
  // Staging for updates: a ring of pinned slots per update, reused once the
  // frame that read a slot has finished (the Recycler's rule, :296-363).
  for (const UpdateDecl& u : g->updates) {
    UpdateRt ur;
    uint64_t eb = g->res[u.rid - 1].elem_bytes;
    uint64_t base = (uint64_t)g->res[u.rid - 1].buf->ptr;
    if (u.first) {
      ur.dst = base + (uint64_t)(u.first - 1) * eb;
      ur.max_bytes = (uint64_t)(u.last - u.first + 1) * eb;
    } else {
      ur.dst = base;
      ur.max_bytes = resource_bytes(g, u.rid);
    }
    for (int k = 0; k < kStagingSlots; ++k) {
      if (cudaHostAlloc(&ur.staging[k], std::max<uint64_t>(ur.max_bytes, 16), cudaHostAllocDefault) != cudaSuccess ||
          cudaEventCreateWithFlags(&ur.ev[k], cudaEventDisableTiming) != cudaSuccess) {
        pl->upd.push_back(ur);
        fail(MTL_ERR_OOM, "Update: pinned staging of %llu bytes", (unsigned long long)ur.max_bytes);
        return cleanup(MTL_ERR_OOM);
      }
    }
    pl->upd.push_back(ur);
  }
  if (pl->o.profile) {
    const int n = (int)pl->a.order.size();
    pl->ev_start.resize(n);
    pl->ev_end.resize(n);
    pl->gpu_ms.assign(n, {});
    pl->host_ms.assign(n, {});
    for (int p = 0; p < n; ++p)
      if (cudaEventCreate(&pl->ev_start[p]) != cudaSuccess || cudaEventCreate(&pl->ev_end[p]) != cudaSuccess) {
        fail(MTL_ERR_CUDA, "Plan: profiler events");
        return cleanup(MTL_ERR_CUDA);
      }
  }
  if ((st = build_mode(pl, 0))) return cleanup(st);
  *out = pl;
  return MTL_OK;
}

mtl_status mtl_plan_release(mtl_plan* pl) {
  plan_free(pl);
  return MTL_OK;
}

mtl_status mtl_plan_run(mtl_plan* pl, int32_t barriers) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "run!: plan is NULL");
  if (barriers < MTL_BARRIERS_DERIVED || barriers > MTL_BARRIERS_BOTH)
    return fail(MTL_ERR_ARGUMENT, "barriers must be :derived, :backend or :both, got %d", barriers);
  if (!pl->g->dev) return fail(MTL_ERR_STATE, "run!: this plan was compiled without a device");
  if (mtl_status s = injected("mtl_plan_run")) return s;
  mtl_device* d = pl->g->dev;
  if (mtl_status s = use_device(d)) return s;
  // :both is the derived edges together with the serial chain, which is the
  // serial chain.
  const int mode = barriers == MTL_BARRIERS_DERIVED ? 0 : 1;
  if (mtl_status s = build_mode(pl, mode)) return s;
  ModeGraph& m = pl->modes[mode];
  collect(pl);
  if (m.direct) return m.direct(d->stream);

  auto t0 = std::chrono::steady_clock::now();
  std::vector<int> used_slot(pl->upd.size(), -1);
  for (size_t u = 0; u < pl->upd.size(); ++u) {
    UpdateRt& ur = pl->upd[u];
    int want_host = 0, want_dev = 0;
    if (ur.pending) {
      if (ur.pending_dev) {
        CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(m.exec, m.upd_dev[u], (void*)ur.dst, ur.pending,
                                                    ur.pending_bytes, cudaMemcpyDeviceToDevice));
        want_dev = 1;
      } else if (ur.pending_pinned) {
        // The caller's page-locked memory is read by DMA as the frame runs;
        // Update retains it, as the reference's ref(x) retains x.
        CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(m.exec, m.upd_host[u], (void*)ur.dst, ur.pending,
                                                    ur.pending_bytes, cudaMemcpyHostToDevice));
        want_host = 1;
      } else {
        int k = ur.next;
        ur.next = (ur.next + 1) % kStagingSlots;
        if (ur.ev_used[k]) CUDA_TRY(cudaEventSynchronize(ur.ev[k]));
        memcpy(ur.staging[k], ur.pending, ur.pending_bytes);
        CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(m.exec, m.upd_host[u], (void*)ur.dst, ur.staging[k],
                                                    ur.pending_bytes, cudaMemcpyHostToDevice));
        used_slot[u] = k;
        want_host = 1;
      }
      ur.pending = nullptr;
    }
    if (m.upd_host_on[u] != want_host) {
      CUDA_TRY(cudaGraphNodeSetEnabled(m.exec, m.upd_host[u], want_host));
      m.upd_host_on[u] = (int8_t)want_host;
    }
    if (m.upd_dev_on[u] != want_dev) {
      CUDA_TRY(cudaGraphNodeSetEnabled(m.exec, m.upd_dev[u], want_dev));
      m.upd_dev_on[u] = (int8_t)want_dev;
    }
  }
  double host_update_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();

  CUDA_TRY(cudaGraphLaunch(m.exec, d->stream));
  for (size_t u = 0; u < pl->upd.size(); ++u)
    if (used_slot[u] >= 0) {
      CUDA_TRY(cudaEventRecord(pl->upd[u].ev[used_slot[u]], d->stream));
      pl->upd[u].ev_used[used_slot[u]] = true;
    }
  if (pl->o.profile) {
    pl->prof_pending = true;
    pl->prof_mode = mode;
    for (size_t p = 0; p < pl->a.order.size(); ++p) {
      const Pass& ps = pl->g->passes[pl->a.order[p]];
      sample(pl->host_ms[p], ps.kind == MTL_PASS_UPDATE ? host_update_ms : 0.0);
    }
  }
  return MTL_OK;
}

mtl_status mtl_plan_update(mtl_plan* pl, int32_t update, const void* data, uint64_t bytes,
                           int32_t data_on_device) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "Update: plan is NULL");
  if (update < 0 || update >= (int)pl->upd.size()) return fail(MTL_ERR_ARGUMENT, "Update: no update %d", update);
  UpdateRt& ur = pl->upd[update];
  if (!data || bytes == 0) return fail(MTL_ERR_ARGUMENT, "Update: empty data");
  const UpdateDecl& ud = pl->g->updates[update];
  if (ud.first ? bytes != ur.max_bytes : bytes > ur.max_bytes)
    return fail(MTL_ERR_ARGUMENT, "Update: %llu bytes of data for a %s of %llu bytes", (unsigned long long)bytes,
                ud.first ? "range" : "buffer", (unsigned long long)ur.max_bytes);
  ur.pending = data;
  ur.pending_bytes = bytes;
  ur.pending_dev = data_on_device != 0;
  ur.pending_pinned = false;
  if (!ur.pending_dev && pl->g->dev) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, data) == cudaSuccess && at.type == cudaMemoryTypeHost)
      ur.pending_pinned = true;
    cudaGetLastError();
  }
  return MTL_OK;
}

mtl_status mtl_plan_set_arg(mtl_plan* pl, int32_t pass, int32_t dispatch, int32_t index,
                            const mtl_arg* arg) {
  if (!pl || !arg) return fail(MTL_ERR_ARGUMENT, "set_arg: NULL argument");
  mtl_graph* g = pl->g;
  if (pass < 0 || pass >= (int)g->passes.size()) return fail(MTL_ERR_ARGUMENT, "set_arg: no pass %d", pass);
  Pass& ps = g->passes[pass];
  if (dispatch < 0 || dispatch >= (int)ps.dispatches.size())
    return fail(MTL_ERR_ARGUMENT, "set_arg: pass \"%s\" has no dispatch %d", ps.name.c_str(), dispatch);
  Dispatch& d = ps.dispatches[dispatch];
  if (index < 0 || index >= (int)d.args.size()) return fail(MTL_ERR_ARGUMENT, "set_arg: no argument %d", index);
  mtl_arg& cur = d.args[index];
  if (cur.kind == MTL_ARG_RESOURCE || cur.kind == MTL_ARG_PTR || cur.kind != arg->kind)
    return fail(MTL_ERR_ARGUMENT, "set_arg: only a scalar argument can change, and only to the same type");
  cur = *arg;
  if (!g->dev) return MTL_OK;
  if (mtl_status s = use_device(g->dev)) return s;
  const int pos = position_of(pl, pass);
  const bool fused = pos >= 0 && compiled_step(pl, pos);
  for (auto& m : pl->modes) {
    if (!m.built || pos < 0) continue;
    cudaGraph_t child = nullptr;
    if (mtl_status s = fused ? capture_fused(pl, pos, &child) : capture_dispatch(pl, d, &child)) return s;
    cudaError_t e = cudaGraphExecChildGraphNodeSetParams(m.exec, m.dispatch_nodes[pos][fused ? 0 : dispatch], child);
    cudaGraphDestroy(child);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "set_arg: %s", cudaGetErrorString(e));
    if (m.direct)
      if (mtl_status s = direct_launcher(pl, m, &m.direct)) return s;
  }
  return MTL_OK;
}

// ── plan queries ────────────────────────────────────────────────────────────
mtl_status mtl_plan_npasses(mtl_plan* pl, int32_t* n) {
  if (!pl || !n) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  *n = (int32_t)pl->a.order.size();
  return MTL_OK;
}

mtl_status mtl_plan_order(mtl_plan* pl, int32_t* order, int32_t cap) {
  if (!pl || !order) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  for (int32_t i = 0; i < cap && i < (int32_t)pl->a.order.size(); ++i) order[i] = pl->a.order[i];
  return MTL_OK;
}

static mtl_status copy_ts(const std::vector<Transition>& ts, mtl_transition* out, int32_t cap, int32_t* n) {
  if (n) *n = (int32_t)ts.size();
  for (int32_t i = 0; i < (int32_t)ts.size() && i < cap; ++i) {
    const Transition& t = ts[i];
    if (t.waits.size() > MTL_MAX_WAITS) return fail(MTL_ERR_UNSUPPORTED, "too many waits");
    out[i].resource = t.resource;
    out[i].from = t.from;
    out[i].to = t.to;
    out[i].nwaits = (int32_t)t.waits.size();
    for (size_t k = 0; k < t.waits.size(); ++k) out[i].waits[k] = t.waits[k];
  }
  return MTL_OK;
}

mtl_status mtl_plan_transitions(mtl_plan* pl, int32_t position, mtl_transition* out, int32_t cap, int32_t* n) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "NULL plan");
  if (position < 0 || position >= (int)pl->a.prepass.size()) return fail(MTL_ERR_ARGUMENT, "no position %d", position);
  return copy_ts(pl->a.prepass[position], out, cap, n);
}

mtl_status mtl_plan_edges(mtl_plan* pl, int32_t position, int32_t* preds, int32_t cap, int32_t* n) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "NULL plan");
  if (position < 0 || position >= (int)pl->a.edges.size()) return fail(MTL_ERR_ARGUMENT, "no position %d", position);
  const auto& e = pl->a.edges[position];
  if (n) *n = (int32_t)e.size();
  for (int32_t i = 0; i < cap && i < (int32_t)e.size(); ++i) preds[i] = e[i] - 1;  // 0-based positions
  return MTL_OK;
}

mtl_status mtl_plan_deps(mtl_plan* pl, int32_t pass, int32_t* deps, int32_t cap, int32_t* n) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "NULL plan");
  if (pass < 0 || pass >= (int)pl->a.deps.size()) return fail(MTL_ERR_ARGUMENT, "no pass %d", pass);
  const auto& e = pl->a.deps[pass];
  if (n) *n = (int32_t)e.size();
  for (int32_t i = 0; i < cap && i < (int32_t)e.size(); ++i) deps[i] = e[i];
  return MTL_OK;
}

mtl_status mtl_plan_peakbytes(mtl_plan* pl, int64_t* peak) {
  if (!pl || !peak) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  *peak = pl->a.peak;
  return MTL_OK;
}

mtl_status mtl_plan_naivebytes(mtl_plan* pl, int64_t* naive) {
  if (!pl || !naive) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  *naive = pl->a.naive;
  return MTL_OK;
}

mtl_status mtl_plan_offset(mtl_plan* pl, int32_t index, int64_t* offset) {
  if (!pl || !offset) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  if (index < 0 || index >= (int)pl->a.offsets.size()) return fail(MTL_ERR_ARGUMENT, "no transient %d", index);
  *offset = pl->a.offsets[index];
  return MTL_OK;
}

mtl_status mtl_plan_ntransients(mtl_plan* pl, int32_t* n) {
  if (!pl || !n) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  *n = (int32_t)pl->a.offsets.size();
  return MTL_OK;
}

mtl_status mtl_plan_resource_ptr(mtl_plan* pl, int32_t rid, void** ptr) {
  if (!pl || !ptr) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  if (rid < 1 || rid > (int)pl->g->res.size()) return fail(MTL_ERR_ARGUMENT, "no resource %d", rid);
  if (!pl->g->dev) return fail(MTL_ERR_STATE, "plan has no device");
  *ptr = (void*)resource_ptr(pl, rid);
  return MTL_OK;
}

mtl_status mtl_plan_nkernels(mtl_plan* pl, int32_t barriers, int32_t* n) {
  if (!pl || !n) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  int mode = barriers == MTL_BARRIERS_DERIVED ? 0 : 1;
  if (!pl->g->dev) return fail(MTL_ERR_STATE, "plan has no device");
  if (mtl_status s = use_device(pl->g->dev)) return s;
  if (mtl_status s = build_mode(pl, mode)) return s;
  *n = pl->modes[mode].nkernels;
  return MTL_OK;
}

mtl_status mtl_plan_nedges(mtl_plan* pl, int32_t barriers, int32_t* n) {
  if (!pl || !n) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  if (barriers == MTL_BARRIERS_DERIVED) {
    int e = 0;
    for (auto& v : pl->a.edges) e += (int)v.size();
    *n = e;
  } else {
    *n = std::max<int>(0, (int)pl->a.order.size() - 1);
  }
  return MTL_OK;
}

mtl_status mtl_plan_timings(mtl_plan* pl, mtl_timing* out, int32_t cap, int32_t* n) {
  if (!pl) return fail(MTL_ERR_ARGUMENT, "NULL plan");
  if (!pl->o.profile)
    return fail(MTL_ERR_ARGUMENT, "timings: this plan was built without profile = true");
  collect(pl);
  const int np = (int)pl->a.order.size();
  if (n) *n = np;
  for (int p = 0; p < np && p < cap; ++p) {
    const Pass& ps = pl->g->passes[pl->a.order[p]];
    memset(&out[p], 0, sizeof(mtl_timing));
    std::string name = ps.name;  // a fused run is named by its members, joined by '+'
    for (size_t k = 1; k < pl->a.steps[p].size(); ++k) name += "+" + pl->g->passes[pl->a.steps[p][k]].name;
    snprintf(out[p].name, sizeof out[p].name, "%s", name.c_str());
    out[p].kind = ps.kind;
    out[p].samples = (int32_t)pl->gpu_ms[p].size();
    out[p].gpu_ms = median(pl->gpu_ms[p]);
    out[p].host_ms = median(pl->host_ms[p]);
  }
  return MTL_OK;
}

// ── direct launches ─────────────────────────────────────────────────────────
static mtl_status direct_args(int32_t kernel, const mtl_arg* args, int32_t nargs, const int64_t* nd,
                              int32_t ndim, LaunchArgs& la) {
  const KernelDesc* kd = kernel_desc(kernel);
  if (!kd) return fail(MTL_ERR_ARGUMENT, "unknown kernel %d", kernel);
  if (nargs != (int)strlen(kd->sig))
    return fail(MTL_ERR_ARGUMENT, "%s takes %zu arguments (%s), got %d", kd->name, strlen(kd->sig), kd->sig, nargs);
  if (ndim < 1 || ndim > 3 || !nd) return fail(MTL_ERR_ARGUMENT, "ndrange must have 1-3 dimensions");
  la.ndim = ndim;
  for (int i = 0; i < 3; ++i) la.nd[i] = i < ndim ? nd[i] : 1;
  for (int i = 0; i < ndim; ++i)
    if (nd[i] < 0) return fail(MTL_ERR_ARGUMENT, "negative ndrange");
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  la.sm_count = sms;
  la.device = dev;
  for (int i = 0; i < nargs; ++i) {
    Arg x;
    const mtl_arg& m = args[i];
    switch (m.kind) {
      case MTL_ARG_PTR: x.kind = MTL_ARG_PTR; x.ptr = m.v.ptr; x.bytes = m.bytes; break;
      case MTL_ARG_F32: x.kind = m.kind; x.f32 = m.v.f32; break;
      case MTL_ARG_I32: x.kind = m.kind; x.i32 = m.v.i32; break;
      case MTL_ARG_I64: x.kind = m.kind; x.i64 = m.v.i64; break;
      case MTL_ARG_F64: x.kind = m.kind; x.f64 = m.v.f64; break;
      case MTL_ARG_NULL: x.kind = MTL_ARG_NULL; break;
      default: return fail(MTL_ERR_ARGUMENT, "%s: argument %d is a graph resource; direct launches take pointers", kd->name, i + 1);
    }
    char c = kd->sig[i];
    bool ok = (c == 'B' && x.kind == MTL_ARG_PTR) || (c == 'b' && (x.kind == MTL_ARG_PTR || x.kind == MTL_ARG_NULL)) ||
              (c == 'f' && x.kind == MTL_ARG_F32) || (c == 'i' && x.kind == MTL_ARG_I32) ||
              (c == 'I' && x.kind == MTL_ARG_I64) || (c == 'd' && x.kind == MTL_ARG_F64);
    if (!ok) return fail(MTL_ERR_ARGUMENT, "%s: argument %d has the wrong kind (%s)", kd->name, i + 1, kd->sig);
    la.a.push_back(x);
  }
  return MTL_OK;
}

mtl_status mtl_kernel_workspace(int32_t kernel, const mtl_arg* args, int32_t nargs, const int64_t* nd,
                                int32_t ndim, uint64_t* bytes) {
  if (!bytes) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  LaunchArgs la;
  if (mtl_status s = direct_args(kernel, args, nargs, nd, ndim, la)) return s;
  const KernelDesc* kd = kernel_desc(kernel);
  *bytes = kd->workspace ? kd->workspace(la) : 0;
  return MTL_OK;
}

mtl_status mtl_launch(int32_t kernel, const mtl_arg* args, int32_t nargs, const int64_t* nd, int32_t ndim,
                      void* workspace, uint64_t workspace_bytes, void* stream) {
  if (mtl_status s = injected("mtl_launch")) return s;
  LaunchArgs la;
  if (mtl_status s = direct_args(kernel, args, nargs, nd, ndim, la)) return s;
  return launch_kernel(kernel, la, workspace, workspace_bytes, stream);
}

}  // extern "C"
