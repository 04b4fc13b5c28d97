// Internal structures shared by the graph compiler (mtl_graph.cpp), the CUDA
// runtime (mtl_runtime.cu) and the kernel registry (kernels/*.cu).
#pragma once

#include <cstdint>
#include <cstdio>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/mantle_cuda.h"

namespace mtl {

// ── errors ──────────────────────────────────────────────────────────────────
// Thread-local message for mtl_last_error(); every entry point returns a status.
void set_error(const char* fmt, ...);
mtl_status fail(mtl_status st, const char* fmt, ...);
// Returns MTL_ERR_INJECTED (and records why) when a failure was injected for
// this entry point; MTL_OK otherwise.
mtl_status injected(const char* entry_point);

// ── usage vocabulary (src/sync/usage.jl:120-167) ────────────────────────────
inline uint32_t base_of(uint32_t u) { return u & MTL_U_BASE_MASK; }
inline bool is_unordered(uint32_t u) { return (u & MTL_U_UNORDERED) != 0; }
inline uint32_t inner_of(uint32_t u) { return u & ~uint32_t(MTL_U_UNORDERED); }
bool usage_reads(uint32_t u);
bool usage_writes(uint32_t u);
bool usage_discards(uint32_t u);
bool usage_valid(uint32_t u);
bool needs_transition(int backend, int kind, uint32_t before, uint32_t after);

struct Transition {
  int resource = 0;
  uint32_t from = 0;
  std::vector<uint32_t> waits;
  uint32_t to = 0;
};

// Per-resource tracking state (src/sync/transition.jl:36-43): `current` is the
// usage the resource is in (0 = nothing), `pending` the reads since the last
// write.
struct ResourceState {
  uint32_t current = 0;
  std::vector<uint32_t> pending;
};

// transition!(out, backend, resource, state, next): transition.jl:79-92.
// Returns true when a transition was appended.
bool transition_step(std::vector<Transition>& out, int backend, int kind, int resource,
                     ResourceState& st, uint32_t next);

// ── memory placement (src/memory/*.jl) ─────────────────────────────────────
struct Gap {
  int64_t lower, upper;
  bool has_window;
  int64_t wlo, whi;
};
struct Item {
  std::string id;
  int64_t lower, upper;  // half-open
  int64_t size;
  int64_t alignment = 1;
  int64_t offset = -1;  // pinned when >= 0
  std::vector<Gap> gaps;
};
struct Placement {
  std::vector<int64_t> offsets;  // per item, input order
  int64_t height = 0;
};
mtl_status place(const std::vector<Item>& items, int strategy, Placement& out);
int64_t maxload(const std::vector<Item>& items);

// ── kernels ─────────────────────────────────────────────────────────────────
// A resolved argument: a device pointer or a scalar.
struct Arg {
  int kind = MTL_ARG_NULL;  // MTL_ARG_PTR after resolution, or a scalar kind
  uint64_t ptr = 0;
  float f32 = 0;
  int32_t i32 = 0;
  int64_t i64 = 0;
  double f64 = 0;
  int rid = 0;  // the graph resource a PTR came from (0 = none)
  uint64_t bytes = 0;  // size behind a PTR (0 = unknown)
};
struct LaunchArgs {
  std::vector<Arg> a;
  int64_t nd[3] = {1, 1, 1};
  int ndim = 1;
  int group[3] = {0, 0, 0};
  int sm_count = 148;
  int device = -1;  // CUDA ordinal the launch is for (-1: none, shapes use sm_count)
};

// Description of one elementwise micro-op program (fused chains). Defined in
// kernels/elementwise.cu; the compiler only needs to know whether a kernel is
// elementwise and how to splice its program.
struct EwOp {
  uint8_t op, dst, a, b, c;
  float imm;
};
enum EwOpcode : uint8_t {
  EW_MOV = 0,
  EW_ADD,
  EW_SUB,
  EW_MUL,
  EW_FMA,
  EW_ABS,
  EW_SQRT,
  EW_SIN,
  EW_MULK,  // a * imm
  EW_ADDK,  // a + imm
  EW_CONST  // imm
};

struct KernelDesc {
  const char* name;
  // One char per argument: B buffer (pointer), b nullable buffer, f f32, i i32,
  // I i64, d f64.
  const char* sig;
  // Elementwise kernels: element i of every buffer argument depends only on
  // element i of the inputs, so consecutive ones may be fused.
  bool elementwise;
  // Which buffer arguments are read / written (bit per argument index).
  uint32_t reads_mask;
  uint32_t writes_mask;
  // Checks the launch against the sizes of its buffer arguments (bytes[i], 0 =
  // unknown) so that nothing is launched that could touch memory out of bounds.
  mtl_status (*check)(const LaunchArgs&, const uint64_t* bytes);
  uint64_t (*workspace)(const LaunchArgs&);
  // Non-elementwise kernels launch through this; elementwise ones run through
  // the micro-op interpreter.
  mtl_status (*launch)(const LaunchArgs&, void* ws, uint64_t ws_bytes, void* stream);
  // Elementwise kernels only: append this dispatch's micro-ops. `slot` maps an
  // argument index to a register already holding that argument's value (-1 =
  // none); returns the register of each written argument through `out_reg`.
  int (*ew_emit)(const LaunchArgs&, std::vector<EwOp>& prog, int* slot, int* out_reg,
                 int* nregs);
};
const KernelDesc* kernel_desc(int id);
int kernel_count();
int kernel_find(const char* name);

// Launch the fused elementwise program (kernels/elementwise.cu).
struct EwProgram {
  std::vector<uint64_t> inputs;   // device pointers, loaded into registers 0..nin-1
  std::vector<uint64_t> outputs;  // device pointers
  std::vector<int> out_regs;      // register stored to each output
  std::vector<EwOp> ops;
  int nregs = 0;
  int64_t n = 0;
};
mtl_status ew_launch_program(const EwProgram& p, void* stream);
struct EwMember {
  const KernelDesc* kd;
  LaunchArgs la;
};
mtl_status ew_build_program(const std::vector<EwMember>& ms, const std::vector<uint64_t>& elided,
                            EwProgram& out);
mtl_status ew_launch_single(const KernelDesc* kd, const LaunchArgs& la, void* stream);
// Whether a built program is within the limits of the fused kernel.
bool ew_program_fits(const EwProgram& p);
// Whether pass `pid` of a graph can be run as a compiled elementwise program:
// one elementwise dispatch over a 1-D range whose arguments are whole declared
// resources (the passes a fused run may hold).
bool mtl_pass_compilable(const ::mtl_graph* g, int pid);
// A program compiled to a straight-line kernel (kernels/ew_compile.cu): compile
// (cached; outside stream capture) and launch.
mtl_status ew_compile(const EwProgram& p, void** kernel);
mtl_status ew_launch_compiled(void* kernel, const EwProgram& p, void* stream);
// Validates and launches any built-in kernel (elementwise or not).
mtl_status launch_kernel(int kernel, const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream);

// ── graph model ─────────────────────────────────────────────────────────────
enum ResKind { RES_PERSISTENT = 0, RES_TRANSIENT = 1, RES_VIEW = 2 };

struct Resource {
  int kind = RES_PERSISTENT;
  uint64_t elems = 0;
  uint32_t elem_bytes = 4;
  int parent = 0;                // views: the buffer they slice
  int64_t first = 0, last = 0;   // views: 1-based inclusive element range
  mtl_buffer* buf = nullptr;     // persistent
  int transient_index = -1;      // transients: index in Graph::transients
  bool internal = false;         // workspace the compiler added for a kernel
};

struct Transient {
  int rid = 0;
  int64_t first = 0, last = 0;  // scheduled positions (1-based), from Liveness
  uint64_t bytes = 0;
  int64_t alignment = 256;
};

struct Dispatch {
  int kernel = -1;
  std::vector<mtl_arg> args;
  int64_t nd[3] = {1, 1, 1};
  int ndim = 1;
  int group[3] = {0, 0, 0};
  int workspace_rid = 0;  // internal transient holding the kernel's scratch
};

struct UpdateDecl {
  int rid = 0;
  int64_t first = 0, last = 0;  // 0 = whole buffer
};

struct Pass {
  std::string name;
  int kind = MTL_PASS_COMPUTE;
  std::vector<std::pair<int, uint32_t>> usages;
  std::vector<Dispatch> dispatches;
  mtl_custom_fn custom_fn = nullptr;
  void* custom_user = nullptr;
  int copy_src = 0, copy_dst = 0;
};

// Result of the compile phases (src/phases.jl:90), host-only.
struct Analysis {
  std::vector<std::vector<int>> deps;  // Dag: per pass, earlier passes it depends on
  std::vector<int> order;              // Schedule: pass indices in execution order
  std::vector<Item> items;             // Liveness
  std::vector<int64_t> offsets;        // Place: per transient
  int64_t peak = 0, naive = 0;
  std::map<int, std::vector<std::pair<int, int>>> alias_begins;  // Aliasing
  std::vector<std::vector<Transition>> prepass;  // Barriers, per scheduled position
  std::vector<Transition> transitions;
  // Lowering: per scheduled position, the positions whose completion it waits on.
  std::vector<std::vector<int>> edges;
  // Per scheduled position, the passes it runs (more than one: a fused run).
  std::vector<std::vector<int>> steps;
  // Transients a fused run keeps in registers: no storage, never stored.
  std::vector<int> elided;
  std::map<int, std::vector<int>> segments;  // resource id -> atomic segment ids
};

}  // namespace mtl

struct mtl_graph {
  int refs = 1;  // the handle's own reference + one per plan
  mtl_device* dev = nullptr;
  std::vector<mtl::Resource> res;  // index = rid - 1
  std::vector<mtl::Transient> transients;
  std::vector<mtl::Pass> passes;
  std::vector<mtl::UpdateDecl> updates;
  int update_pass = -1;
  std::map<std::pair<int, std::pair<int64_t, int64_t>>, int> views;
  std::map<mtl_buffer*, int> persistent_ids;
};

namespace mtl {
// Lifetimes. Handles reference what they use — a graph its device and the
// buffers it names, a plan its graph, a buffer its device — so the owner's
// release call (Python finalizers, Julia finalizers) may come in any order;
// the object is freed when its last reference goes.
void retain_device(mtl_device* d);
void release_device(mtl_device* d);
void retain_buffer(mtl_buffer* b);
void release_buffer(mtl_buffer* b);
void retain_graph(mtl_graph* g);
void release_graph(mtl_graph* g);

struct CompileOpts {
  bool alias = true, coalesce = true, profile = false, fuse = false;
  int policy = MTL_POLICY_OVERLAP;
};
// Runs Dag, Schedule, Liveness, Place, Aliasing, Barriers and the edge lowering.
mtl_status analyze(mtl_graph* g, const CompileOpts& o, Analysis& a);
bool overlapping(const mtl_graph* g, int a, int b);
// SM count and ordinal of a device (148 / -1 when there is none: analysis-only graphs).
int device_sm_count(mtl_device* d);
int device_ordinal(mtl_device* d);
}  // namespace mtl
