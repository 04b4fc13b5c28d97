/*
 * mantle_cuda.h — C ABI of the B200 execution backend for Mantle.jl.
 *
 * Every entry point returns an mtl_status (0 = MTL_OK). On failure the
 * thread-local text returned by mtl_last_error() says what went wrong; CUDA and
 * NCCL errors are mapped to a status, never abort()ed. Handles are opaque.
 *
 * Each declaration names the reference interface it stands in for
 * (file:line inside SimonDanisch/Mantle.jl). A Julia extension binds these with
 * `ccall`; the Python package `mantle_cuda` binds them with ctypes.
 */
#ifndef MANTLE_CUDA_H
#define MANTLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTL_ABI_VERSION 1

typedef int32_t mtl_status;
enum {
  MTL_OK = 0,
  MTL_ERR_ARGUMENT = 1,    /* ArgumentError in the reference */
  MTL_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  MTL_ERR_STATE = 3,       /* call not valid in this state (e.g. no device) */
  MTL_ERR_OOM = 4,         /* allocation failed or pool cap exceeded */
  MTL_ERR_UNSUPPORTED = 5, /* shape or feature this build does not cover */
  MTL_ERR_TIMEOUT = 6,     /* a bounded device-side wait gave up */
  MTL_ERR_NCCL = 7,        /* a collective failed or was aborted */
  MTL_ERR_INJECTED = 8     /* failure injected on the host for testing */
};

typedef struct mtl_device mtl_device;
typedef struct mtl_buffer mtl_buffer;
typedef struct mtl_graph mtl_graph;
typedef struct mtl_plan mtl_plan;
typedef struct mtl_comm mtl_comm;

/* ── usage vocabulary ────────────────────────────────────────────────────────
 * One 32-bit code per usage: a base kind in the low 5 bits plus flags.
 * Replaces the usage types of src/sync/usage.jl:22-167. `reads`, `writes`,
 * `discards`, `unordered` and `inner` follow usage.jl:120-167 exactly. */
enum {
  MTL_U_STORAGE = 1,     /* Storage{K,Access{rd,wr}}   usage.jl:75  */
  MTL_U_COPY_SRC = 2,    /* CopySrc                    usage.jl:56  */
  MTL_U_COPY_DST = 3,    /* CopyDst                    usage.jl:57  */
  MTL_U_INDIRECT = 4,    /* Indirect                   usage.jl:52  */
  MTL_U_UNIFORM = 5,     /* Uniform                    usage.jl:53  */
  MTL_U_VERTICES = 6,    /* Vertices                   usage.jl:50  */
  MTL_U_INDICES = 7,     /* Indices                    usage.jl:51  */
  MTL_U_SAMPLED = 8,     /* Sampled                    usage.jl:54  */
  MTL_U_PRESENT = 9,     /* Present                    usage.jl:55  */
  MTL_U_TRACE_READ = 10, /* TraceRead                  usage.jl:58  */
  MTL_U_TRACE_BUILD = 11,/* TraceBuild                 usage.jl:59  */
  MTL_U_COLOR = 12,      /* ColorAttachment{Discard}   usage.jl:84  */
  MTL_U_DEPTH = 13,      /* Depth{DA,SA,Discard}       usage.jl:99 */
  MTL_U_UNDEFINED = 14,  /* Undefined                  usage.jl:70  */
  MTL_U_BASE_MASK = 0x1f,
  MTL_U_READ = 1 << 5,          /* Access read bit (Storage; depth aspect) */
  MTL_U_WRITE = 1 << 6,         /* Access write bit                        */
  MTL_U_STENCIL_READ = 1 << 7,  /* Depth stencil aspect; neither = NoAccess */
  MTL_U_STENCIL_WRITE = 1 << 8,
  MTL_U_DISCARD = 1 << 9,       /* load op discards (Color/Depth)          */
  MTL_U_IMAGE = 1 << 10,        /* Storage{ImageKind,…}; else BufferKind   */
  MTL_U_UNORDERED = 1 << 11     /* Unordered{U}              usage.jl:159  */
};

/* Property queries over a usage code (usage.jl:120-167). */
int32_t mtl_usage_reads(uint32_t usage);
int32_t mtl_usage_writes(uint32_t usage);
int32_t mtl_usage_discards(uint32_t usage);

enum { MTL_KIND_BUFFER = 0, MTL_KIND_IMAGE = 1, MTL_KIND_ACCEL = 2 };
enum { MTL_BACKEND_CUDA = 0, MTL_BACKEND_WEBGPU = 1 };

/* A transition as src/sync/transition.jl:16-21 defines it. `resource` 0 is an
 * aliasing handover (ext/MantleLavaExt.jl:1793-1806). */
#define MTL_MAX_WAITS 16
typedef struct mtl_transition {
  int32_t resource;
  uint32_t from;
  uint32_t to;
  int32_t nwaits;
  uint32_t waits[MTL_MAX_WAITS];
} mtl_transition;

/* needs_transition(backend, kind, before, after): the portable rule of
 * src/sync/transition.jl:56-66; WebGPU never needs one (sync/backend.jl:22). */
int32_t mtl_needs_transition(int32_t backend, int32_t kind, uint32_t before, uint32_t after);

/* transitions(backend, kind, usages; initial): src/sync/transition.jl:103-111.
 * `initial` 0 = nothing. Writes at most `cap` transitions, count in *n. */
mtl_status mtl_transitions(int32_t backend, int32_t kind, const uint32_t* usages, int32_t nusages,
                           uint32_t initial, mtl_transition* out, int32_t cap, int32_t* n);

/* ── memory placement (src/memory/*.jl) ───────────────────────────────────── */
typedef struct mtl_gap {
  int64_t lower, upper;            /* Gap.during, half-open          model.jl:27 */
  int64_t window_lower, window_upper; /* OffsetWindow; lower<0 = nothing */
} mtl_gap;

typedef struct mtl_item {
  int64_t lower, upper;            /* Item.live, half-open Span      model.jl:39-49 */
  int64_t size;
  int64_t alignment;               /* 1 = none */
  int64_t offset;                  /* pinned offset, or -1           model.jl:48-51 */
  int32_t ngaps;
  const mtl_gap* gaps;
  const char* id;                  /* tie-break key, as Item.id      placement.jl:37 */
} mtl_item;

enum { MTL_LOWEST_FIT = 0, MTL_BEST_FIT = 1 };

/* place(problem, strategy): src/memory/placement.jl:46-99. */
mtl_status mtl_place(const mtl_item* items, int32_t n, int32_t strategy, int64_t* offsets,
                     int64_t* height);
/* maxload(problem): src/memory/bound.jl:14-28. */
mtl_status mtl_maxload(const mtl_item* items, int32_t n, int64_t* out);

/* ── errors and library info ─────────────────────────────────────────────── */
const char* mtl_last_error(void);
int32_t mtl_abi_version(void);
/* Host-side fault injection: the next `count` calls of the named entry point
 * (e.g. "mtl_buffer_alloc") fail with MTL_ERR_INJECTED. count 0 clears. */
mtl_status mtl_inject_failure(const char* entry_point, int32_t count);

/* ── device ─────────────────────────────────────────────────────────────── */
/* Mantle.Device(): ext/MantleLavaExt.jl:16-25. One CUDA device and its queue
 * (one stream). `pool_cap_bytes` 0 = no cap on plan slabs. */
mtl_status mtl_device_open(int32_t ordinal, uint64_t pool_cap_bytes, mtl_device** out);
mtl_status mtl_device_close(mtl_device* dev);
mtl_status mtl_device_synchronize(mtl_device* dev);
/* The device's stream (cudaStream_t) — Mantle.backend(dev), src/runtime/api.jl:37-49. */
mtl_status mtl_device_stream(mtl_device* dev, void** stream);
mtl_status mtl_device_info(mtl_device* dev, int32_t* sm_count, int64_t* l2_bytes,
                           int64_t* hbm_bytes, int32_t* cc_major, int32_t* cc_minor);

/* ── persistent buffers ──────────────────────────────────────────────────── */
/* Buffer(dev, T, n) / Buffer(dev, data; capacity): ext/MantleLavaExt.jl:77-88. */
mtl_status mtl_buffer_alloc(mtl_device* dev, uint64_t bytes, mtl_buffer** out);
/* Wrap device memory owned by someone else (a torch tensor, a CuArray). */
mtl_status mtl_buffer_wrap(mtl_device* dev, void* device_ptr, uint64_t bytes, mtl_buffer** out);
/* update!(buf, r, data): ext/MantleLavaExt.jl:103-112 (synchronous on the device stream). */
mtl_status mtl_buffer_upload(mtl_buffer* buf, const void* host, uint64_t offset, uint64_t bytes);
/* Array(buf): ext/MantleLavaExt.jl:122 (synchronises, as a readback must). */
mtl_status mtl_buffer_download(mtl_buffer* buf, void* host, uint64_t offset, uint64_t bytes);
mtl_status mtl_buffer_device_ptr(mtl_buffer* buf, void** ptr);
mtl_status mtl_buffer_release(mtl_buffer* buf);

/* ── graph recording ─────────────────────────────────────────────────────── */
/* Graph(dev): ext/MantleLavaExt.jl:383-386. dev may be NULL: the graph can then
 * be compiled (phases only) but not instantiated — used by the host tests. */
mtl_status mtl_graph_create(mtl_device* dev, mtl_graph** out);
mtl_status mtl_graph_release(mtl_graph* g);

/* A persistent buffer as a graph resource (resourceid, MantleLavaExt.jl:526-530).
 * buf may be NULL for an analysis-only graph. Returns the resource id (>=1). */
mtl_status mtl_graph_persistent(mtl_graph* g, mtl_buffer* buf, uint64_t elems, uint32_t elem_bytes,
                                int32_t* rid);
/* Transient.Buffer(g, T, n): ext/MantleLavaExt.jl:388-392. */
mtl_status mtl_graph_transient(mtl_graph* g, uint64_t elems, uint32_t elem_bytes, int32_t* rid);

enum { MTL_PASS_COMPUTE = 0, MTL_PASS_CUSTOM = 1, MTL_PASS_UPDATE = 2, MTL_PASS_COPY = 3 };

/* compute!(f, g, name) / custom!(f, g, name): ext/MantleLavaExt.jl:744-766. */
mtl_status mtl_graph_pass(mtl_graph* g, const char* name, int32_t kind, int32_t* pass);

/* use(p, x; read, write, range): ext/MantleLavaExt.jl:722-730. `usage` is a code
 * above (MTL_U_STORAGE|MTL_U_READ… for `use`). first/last: 1-based inclusive
 * element range, or first = 0 for the whole resource (slice, :700-710).
 * *out_rid receives the id the usage is tracked under (the slice's id). */
mtl_status mtl_graph_use(mtl_graph* g, int32_t pass, int32_t rid, uint32_t usage, int64_t first,
                         int64_t last, int32_t* out_rid);

/* Kernel arguments. A RESOURCE argument names a graph resource id and resolves
 * to its device address when the plan is instantiated (the kernel receives the
 * whole buffer even when the usage named a slice, MantleLavaExt.jl:679-681).
 * PTR is a raw device address (direct launches). */
enum {
  MTL_ARG_RESOURCE = 0,
  MTL_ARG_PTR = 1,
  MTL_ARG_F32 = 2,
  MTL_ARG_I32 = 3,
  MTL_ARG_I64 = 4,
  MTL_ARG_F64 = 5,
  MTL_ARG_NULL = 6
};
typedef struct mtl_arg {
  int32_t kind;
  int32_t rid;
  union {
    float f32;
    int32_t i32;
    int64_t i64;
    double f64;
    uint64_t ptr;
  } v;
  /* PTR arguments: size of the memory behind the pointer, checked against
   * what the kernel will touch (0 = unknown, the caller vouches for it).
   * RESOURCE arguments are checked against the resource's own size. */
  uint64_t bytes;
} mtl_arg;

/* Built-in sm_100a kernel families a dispatch can name (the AOT replacement of
 * compiling a KernelAbstractions kernel per dispatch, MantleLavaExt.jl:1909-1928).
 * Their names and argument signatures are listed by mtl_kernel_info. */
mtl_status mtl_kernel_lookup(const char* name, int32_t* kernel);
mtl_status mtl_kernel_info(int32_t kernel, const char** name, const char** signature);
int32_t mtl_kernel_count(void);

/* dispatch!(p, kernel, args, ndrange; group): ext/MantleLavaExt.jl:751-752. */
mtl_status mtl_graph_dispatch(mtl_graph* g, int32_t pass, int32_t kernel, const mtl_arg* args,
                              int32_t nargs, const int64_t* ndrange, int32_t ndim,
                              const int32_t* group);

/* custom!: the body runs once per instantiation under stream capture, and the
 * launches it makes on `stream` become a child graph (MantleLavaExt.jl:757-766).
 * `plan` is the plan being instantiated: mtl_plan_resource_ptr(plan, rid) gives
 * the storage of any resource the body declared (storage(a) in the reference).
 * A non-zero return aborts the instantiation. */
typedef int32_t (*mtl_custom_fn)(void* user, void* stream, mtl_plan* plan);
mtl_status mtl_graph_custom(mtl_graph* g, int32_t pass, mtl_custom_fn fn, void* user);

/* copy!(g, name, dst, src): ext/MantleLavaExt.jl:934-943. */
mtl_status mtl_graph_copy(mtl_graph* g, const char* name, int32_t dst_rid, int32_t src_rid,
                          int32_t* pass);

/* Update(g, buf; range): ext/MantleLavaExt.jl:794-802. first = 0 for the whole
 * buffer. Returns an update handle for mtl_plan_update. */
mtl_status mtl_graph_update(mtl_graph* g, int32_t rid, int64_t first, int64_t last, int32_t* update);

/* ── plan ───────────────────────────────────────────────────────────────── */
enum { MTL_POLICY_OVERLAP = 0, MTL_POLICY_COMPACT = 1 };
typedef struct mtl_plan_opts {
  int32_t coalesce;  /* accepted for API parity; per-resource edges are never coalesced */
  int32_t alias;     /* share transient bytes between disjoint lifetimes */
  int32_t profile;   /* event nodes around every pass, read by mtl_plan_timings */
  int32_t policy;    /* MTL_POLICY_* (src/phases.jl:47-58) */
  int32_t fuse;      /* fuse chains of elementwise dispatches into one kernel */
} mtl_plan_opts;

/* Plan(g; coalesce, alias, profile, policy): ext/MantleLavaExt.jl:1936-1942.
 * Runs Dag, Schedule, Liveness, Place, Aliasing, Barriers (src/phases.jl:90)
 * and, when the graph has a device, lowers the result to a CUDA graph. */
mtl_status mtl_plan_compile(mtl_graph* g, const mtl_plan_opts* opts, mtl_plan** out);
mtl_status mtl_plan_release(mtl_plan* plan);

enum { MTL_BARRIERS_DERIVED = 0, MTL_BARRIERS_BACKEND = 1, MTL_BARRIERS_BOTH = 2 };
/* run!(plan; barriers): ext/MantleLavaExt.jl:2076-2128 — one cudaGraphLaunch on
 * the device's stream; a plan that is a single kernel, with no updates and no
 * profiling, launches that kernel directly on the same stream instead. */
mtl_status mtl_plan_run(mtl_plan* plan, int32_t barriers);

/* UpdateRef(x): ext/MantleLavaExt.jl:776-782. Stores the data for the next
 * run!; a host pointer is copied into a pinned staging slot at run!, a device
 * pointer is copied device to device by the graph. `bytes` must match the
 * declared range (or be <= the buffer for a whole-buffer update). */
mtl_status mtl_plan_update(mtl_plan* plan, int32_t update, const void* data, uint64_t bytes,
                           int32_t data_on_device);

/* Patch a scalar argument of a dispatch (per-frame values such as dt). */
mtl_status mtl_plan_set_arg(mtl_plan* plan, int32_t pass, int32_t dispatch, int32_t index,
                            const mtl_arg* arg);

/* Analysis results (phases), in scheduled order. */
mtl_status mtl_plan_npasses(mtl_plan* plan, int32_t* n);
mtl_status mtl_plan_order(mtl_plan* plan, int32_t* order, int32_t cap);
mtl_status mtl_plan_transitions(mtl_plan* plan, int32_t position, mtl_transition* out, int32_t cap,
                                int32_t* n);
mtl_status mtl_plan_edges(mtl_plan* plan, int32_t position, int32_t* preds, int32_t cap, int32_t* n);
mtl_status mtl_plan_deps(mtl_plan* plan, int32_t pass, int32_t* deps, int32_t cap, int32_t* n);
/* peakbytes(plan) / naivebytes(plan): ext/MantleLavaExt.jl:1279-1282. */
mtl_status mtl_plan_peakbytes(mtl_plan* plan, int64_t* peak);
mtl_status mtl_plan_naivebytes(mtl_plan* plan, int64_t* naive);
/* Offset of transient `index` (creation order) inside the plan slab. */
mtl_status mtl_plan_offset(mtl_plan* plan, int32_t index, int64_t* offset);
mtl_status mtl_plan_ntransients(mtl_plan* plan, int32_t* n);
/* Device address of a resource (persistent, transient or slice) in this plan. */
mtl_status mtl_plan_resource_ptr(mtl_plan* plan, int32_t rid, void** ptr);
/* Kernel nodes in one replay (fused chains count once). */
mtl_status mtl_plan_nkernels(mtl_plan* plan, int32_t barriers, int32_t* n);
mtl_status mtl_plan_nedges(mtl_plan* plan, int32_t barriers, int32_t* n);

/* timings(plan): src/runtime/api.jl:209-241 — per pass in scheduled order. */
typedef struct mtl_timing {
  char name[64];
  int32_t kind;
  int32_t samples;
  double host_ms;
  double gpu_ms;
} mtl_timing;
mtl_status mtl_plan_timings(mtl_plan* plan, mtl_timing* out, int32_t cap, int32_t* n);

/* Resource description, for tests that key transitions by (parent, range). */
mtl_status mtl_graph_resource(mtl_graph* g, int32_t rid, int32_t* kind, int32_t* parent,
                              int64_t* first, int64_t* last, uint64_t* elems);
mtl_status mtl_graph_npasses(mtl_graph* g, int32_t* n);
mtl_status mtl_graph_pass_name(mtl_graph* g, int32_t pass, const char** name);

/* ── direct launches (outside any graph: Mantle.backend(dev), api.jl:37-49) ─ */
/* Launch a built-in kernel on `stream` with PTR/scalar arguments. Kernels that
 * need scratch take it from `workspace` (query the size first). */
mtl_status mtl_kernel_workspace(int32_t kernel, const mtl_arg* args, int32_t nargs,
                                const int64_t* ndrange, int32_t ndim, uint64_t* bytes);
mtl_status mtl_launch(int32_t kernel, const mtl_arg* args, int32_t nargs, const int64_t* ndrange,
                      int32_t ndim, void* workspace, uint64_t workspace_bytes, void* stream);

/* Failure detection for the kernels' bounded waits (no counterpart in the
 * reference, whose Vulkan queue waits are host-side): every spin on an
 * mbarrier in the tensor-core and FFT kernels gives up after a
 * wall-clock limit, records it in a device counter and lets its CTA wind
 * down instead of hanging. *count receives how many CTAs gave up on a wait
 * that ran out (one per CTA, however many of its threads were waiting) on the
 * current device since the last reset; reset != 0 clears the counters. */
mtl_status mtl_kernel_timeouts(int32_t reset, int64_t* count);
/* The wall-clock limit of those waits on the current device, in ns (no
 * counterpart in the reference): 0 restores the default of 2 s; below 1 ms is
 * refused. Tests shorten it to make a wait run out in milliseconds. */
mtl_status mtl_set_wait_limit(uint64_t ns);
/* Test hook for the same failure path (no counterpart in the reference): in
 * the next `launches` launches of the named kernel family ("gemm_bf16" is the
 * one that has the hook) CTA 0's producer issues no load, so that CTA's MMA
 * issuer waits on a stage that never fills until the limit runs out, counts a
 * timeout and winds down with nothing in flight; every other CTA computes its
 * tiles. 0 clears. */
mtl_status mtl_inject_stall(const char* kernel, int32_t launches);

/* Scatter-add / histogram that allocates nothing (no counterpart in the
 * reference). For callers that cannot call cudaMalloc on this path: scratch
 * comes from a fixed MTL_NOALLOC_SCRATCH_BYTES array compiled into the library,
 * held by every GPU that loads it until the process exits. Same arguments and
 * results as the `scatter_add` kernel (acc or hist may be NULL), launched on
 * `stream` for the current device. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) — make it before any stream
 * capture; the lookup is repeated when the call finds another CUDA context
 * current (after cudaDeviceReset, for one), so make the first call after a
 * reset outside a capture too. All calls share the array: calls that overlap
 * on the GPU race, so order them. A call whose bins need more scratch than the
 * array holds fails with MTL_ERR_ARGUMENT. */
#define MTL_NOALLOC_SCRATCH_BYTES (20u << 20)
mtl_status mtl_scatter_add_noalloc(float* acc, uint32_t* hist, const float* values, const int32_t* idx,
                                   int64_t n, int32_t nbins, int32_t accumulate, void* stream);

/* ── collectives (NCCL over NVLink) ──────────────────────────────────────── */
/* One communicator per process/GPU; `unique_id` is NCCL's 128-byte id, shared
 * by the caller over any host channel (torch.distributed's store). */
mtl_status mtl_comm_unique_id(void* unique_id_128);
mtl_status mtl_comm_init(mtl_device* dev, int32_t nranks, int32_t rank, const void* unique_id_128,
                         mtl_comm** out);
mtl_status mtl_comm_release(mtl_comm* comm);
mtl_status mtl_comm_abort(mtl_comm* comm);
/* ncclAllGather of `bytes` per rank, on the device stream. */
mtl_status mtl_allgather(mtl_comm* comm, const void* send, void* recv, uint64_t bytes);
/* How long mtl_comm_init and mtl_allgather wait, on the host, for the
 * communicator before they give up with MTL_ERR_TIMEOUT (the communicator is
 * then aborted): 60 s unless set, process-wide. */
mtl_status mtl_comm_set_timeout(double seconds);

#ifdef __cplusplus
}
#endif
#endif /* MANTLE_CUDA_H */
