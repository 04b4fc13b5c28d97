// Host side of the backend: the usage vocabulary, the per-resource hazard walk,
// the offset placer, graph recording and the compile phases of Mantle.jl
// (src/phases.jl:90) restated in C++, plus the lowering of the derived
// transitions to CUDA-graph dependency edges.
//
// Nothing in this file touches a GPU, so the whole compiler runs (and is
// tested) on a machine without one.

#include <algorithm>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <tuple>

#include "mtl_internal.hpp"

namespace mtl {

// ── errors ──────────────────────────────────────────────────────────────────
static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

mtl_status fail(mtl_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

static std::mutex g_inject_mu;
static std::map<std::string, int> g_inject;

mtl_status injected(const char* entry_point) {
  std::lock_guard<std::mutex> lk(g_inject_mu);
  if (g_inject.empty()) return MTL_OK;
  auto it = g_inject.find(entry_point);
  if (it == g_inject.end() || it->second <= 0) return MTL_OK;
  if (--it->second == 0) g_inject.erase(it);
  return fail(MTL_ERR_INJECTED, "%s: failure injected for testing", entry_point);
}

// ── usage vocabulary ────────────────────────────────────────────────────────
// reads/writes/discards per src/sync/usage.jl:120-144; Unordered forwards to
// its inner usage (usage.jl:166-167).
bool usage_reads(uint32_t u) {
  switch (base_of(u)) {
    case MTL_U_UNDEFINED:
    case MTL_U_COPY_DST:
    case MTL_U_TRACE_BUILD:
      return false;
    case MTL_U_STORAGE:
      return (u & MTL_U_READ) != 0;
    case MTL_U_COLOR:
      return (u & MTL_U_DISCARD) == 0;
    case MTL_U_DEPTH:
      return (u & MTL_U_DISCARD) == 0 && (u & (MTL_U_READ | MTL_U_STENCIL_READ)) != 0;
    default:
      return true;
  }
}

bool usage_writes(uint32_t u) {
  switch (base_of(u)) {
    case MTL_U_COPY_DST:
    case MTL_U_TRACE_BUILD:
    case MTL_U_COLOR:
      return true;
    case MTL_U_STORAGE:
      return (u & MTL_U_WRITE) != 0;
    case MTL_U_DEPTH:
      return (u & (MTL_U_WRITE | MTL_U_STENCIL_WRITE)) != 0;
    default:
      return false;
  }
}

bool usage_discards(uint32_t u) {
  uint32_t b = base_of(u);
  return (b == MTL_U_COLOR || b == MTL_U_DEPTH) && (u & MTL_U_DISCARD) != 0;
}

bool usage_valid(uint32_t u) {
  uint32_t b = base_of(u);
  if (b < MTL_U_STORAGE || b > MTL_U_UNDEFINED) return false;
  if (u & ~uint32_t(0xfff)) return false;
  if (b == MTL_U_STORAGE && (u & (MTL_U_READ | MTL_U_WRITE)) == 0) return false;
  if (b == MTL_U_DEPTH && (u & (MTL_U_READ | MTL_U_WRITE)) == 0) return false;
  return true;
}

// The portable rule, src/sync/transition.jl:56-66: read after read needs
// nothing; two unordered accesses need nothing; anything else involving a
// write does, identical storage writes included. CUDA has no image layouts, so
// this backend uses the portable rule for every resource kind; WebGPU has no
// barriers at all (src/sync/backend.jl:22).
bool needs_transition(int backend, int /*kind*/, uint32_t before, uint32_t after) {
  if (backend == MTL_BACKEND_WEBGPU) return false;
  bool both_unordered = is_unordered(before) && is_unordered(after);
  uint32_t b = inner_of(before), a = inner_of(after);
  if (!usage_writes(b) && !usage_writes(a)) return false;
  if (both_unordered) return false;
  return b != a || usage_writes(b);
}

// transition!, src/sync/transition.jl:79-92.
bool transition_step(std::vector<Transition>& out, int backend, int kind, int resource,
                     ResourceState& st, uint32_t next) {
  uint32_t from = st.current;
  bool emitted = false;
  if (from != 0 && needs_transition(backend, kind, from, next)) {
    Transition t;
    t.resource = resource;
    t.from = from;
    t.to = next;
    if (usage_writes(next)) {
      // unique(vcat(from, pending)), first-appearance order
      t.waits.push_back(from);
      for (uint32_t p : st.pending)
        if (std::find(t.waits.begin(), t.waits.end(), p) == t.waits.end()) t.waits.push_back(p);
    } else {
      t.waits.push_back(from);
    }
    out.push_back(std::move(t));
    st.current = next;
    emitted = true;
  } else if (from == 0) {
    st.current = next;
  }
  if (usage_writes(next))
    st.pending.clear();
  else
    st.pending.push_back(next);
  return emitted;
}

// ── placement (src/memory/placement.jl, bound.jl, model.jl) ─────────────────
static int64_t alignup(int64_t x, int64_t a) { return ((x + a - 1) / a) * a; }

static bool span_overlaps(int64_t al, int64_t au, int64_t bl, int64_t bu) {
  return al < bu && bl < au;
}

// segments(item): the (span, height) pairs an item occupies, gaps applied
// (model.jl:54-65).
struct Seg {
  int64_t lo, hi, h;
};
static std::vector<Seg> segments(const Item& it) {
  std::vector<Seg> out;
  if (it.gaps.empty()) {
    out.push_back({it.lower, it.upper, it.size});
    return out;
  }
  std::vector<Gap> gs = it.gaps;
  std::stable_sort(gs.begin(), gs.end(), [](const Gap& a, const Gap& b) { return a.lower < b.lower; });
  int64_t t = it.lower;
  for (const Gap& g : gs) {
    if (t < g.lower) out.push_back({t, g.lower, it.size});
    if (g.has_window) out.push_back({g.lower, g.upper, g.whi - g.wlo});
    t = g.upper;
  }
  if (t < it.upper) out.push_back({t, it.upper, it.size});
  return out;
}

// conflicts(a, b), placement.jl:7-14.
static bool conflicts(const Item& a, const Item& b) {
  if (!span_overlaps(a.lower, a.upper, b.lower, b.upper)) return false;
  if (a.gaps.empty() && b.gaps.empty()) return true;
  for (const Seg& sa : segments(a))
    for (const Seg& sb : segments(b))
      if (span_overlaps(sa.lo, sa.hi, sb.lo, sb.hi)) return true;
  return false;
}

// priority(i) = (-size, -length(live), id), placement.jl:37.
static bool priority_less(const Item& x, const Item& y) {
  if (x.size != y.size) return x.size > y.size;
  int64_t lx = x.upper - x.lower, ly = y.upper - y.lower;
  if (lx != ly) return lx > ly;
  return x.id < y.id;
}

// place(problem, strategy), placement.jl:46-99.
mtl_status place(const std::vector<Item>& items, int strategy, Placement& out) {
  size_t n = items.size();
  for (const Item& it : items) {
    if (it.lower > it.upper)
      return fail(MTL_ERR_ARGUMENT, "Span(%lld, %lld) is inverted", (long long)it.lower,
                  (long long)it.upper);
    if (it.alignment < 1) return fail(MTL_ERR_ARGUMENT, "item %s: alignment < 1", it.id.c_str());
    if (it.size < 0) return fail(MTL_ERR_ARGUMENT, "item %s: negative size", it.id.c_str());
  }
  std::vector<size_t> pinned, loose;
  for (size_t i = 0; i < n; ++i) (items[i].offset >= 0 ? pinned : loose).push_back(i);
  auto by = [&](size_t a, size_t b) { return priority_less(items[a], items[b]); };
  std::stable_sort(pinned.begin(), pinned.end(), by);
  std::stable_sort(loose.begin(), loose.end(), by);
  std::vector<size_t> order = pinned;
  order.insert(order.end(), loose.begin(), loose.end());

  out.offsets.assign(n, 0);
  out.height = 0;
  std::vector<size_t> settled;
  std::vector<std::pair<int64_t, int64_t>> blocked;
  for (size_t idx : order) {
    const Item& item = items[idx];
    blocked.clear();
    for (size_t j : settled)
      if (conflicts(item, items[j]))
        blocked.push_back({out.offsets[j], out.offsets[j] + items[j].size});
    std::sort(blocked.begin(), blocked.end());
    int64_t off;
    if (item.offset >= 0) {
      off = item.offset;
    } else if (strategy == MTL_BEST_FIT) {
      // choose(::BestFit), placement.jl:89-99
      int64_t best = 0, waste = INT64_MAX, cursor = 0;
      for (auto& [lo, hi] : blocked) {
        if (cursor + item.size <= lo && (lo - cursor) - item.size < waste) {
          best = cursor;
          waste = (lo - cursor) - item.size;
        }
        cursor = std::max(cursor, alignup(hi, item.alignment));
      }
      off = waste == INT64_MAX ? cursor : best;
    } else {
      // choose(::LowestFit), placement.jl:79-86
      off = 0;
      for (auto& [lo, hi] : blocked) {
        if (off + item.size <= lo) break;
        off = std::max(off, alignup(hi, item.alignment));
      }
    }
    for (auto& [lo, hi] : blocked)
      if (off < hi && lo < off + item.size)
        return fail(MTL_ERR_ARGUMENT, "item %s at %lld collides with [%lld, %lld)", item.id.c_str(),
                    (long long)off, (long long)lo, (long long)hi);
    out.offsets[idx] = off;
    settled.push_back(idx);
    out.height = std::max(out.height, off + item.size);
  }
  return MTL_OK;
}

// maxload(problem), bound.jl:14-28: sweep over 2n events.
int64_t maxload(const std::vector<Item>& items) {
  std::vector<std::pair<int64_t, int64_t>> ev;
  for (const Item& it : items)
    for (const Seg& s : segments(it)) {
      if (s.lo == s.hi) continue;
      ev.push_back({s.lo, s.h});
      ev.push_back({s.hi, -s.h});
    }
  if (ev.empty()) return 0;
  std::sort(ev.begin(), ev.end());
  int64_t best = 0, cur = 0;
  for (auto& e : ev) {
    cur += e.second;
    best = std::max(best, cur);
  }
  return best;
}

// ── graph helpers ───────────────────────────────────────────────────────────
static const Resource* res_of(const mtl_graph* g, int rid) {
  if (rid < 1 || rid > (int)g->res.size()) return nullptr;
  return &g->res[rid - 1];
}

// overlapping(g, a, b), ext/MantleLavaExt.jl:1329-1345: equal ids, a slice and
// its parent, or two slices of one parent whose ranges intersect.
bool overlapping(const mtl_graph* g, int a, int b) {
  if (a == b) return true;
  const Resource* ra = res_of(g, a);
  const Resource* rb = res_of(g, b);
  if (!ra || !rb) return false;
  bool va = ra->kind == RES_VIEW, vb = rb->kind == RES_VIEW;
  if (!va && !vb) return false;
  int pa = va ? ra->parent : a;
  int pb = vb ? rb->parent : b;
  if (pa != pb) return false;
  if (!(va && vb)) return true;
  return std::max(ra->first, rb->first) <= std::min(ra->last, rb->last);
}

static int intern_view(mtl_graph* g, int parent, int64_t first, int64_t last) {
  auto key = std::make_pair(parent, std::make_pair(first, last));
  auto it = g->views.find(key);
  if (it != g->views.end()) return it->second;
  Resource r;
  r.kind = RES_VIEW;
  r.parent = parent;
  r.first = first;
  r.last = last;
  const Resource* p = res_of(g, parent);
  r.elem_bytes = p->elem_bytes;
  r.elems = uint64_t(last - first + 1);
  g->res.push_back(r);
  int rid = (int)g->res.size();
  g->views[key] = rid;
  return rid;
}

// The transient a resource id belongs to (itself, or the parent of a slice).
static int transient_of(const mtl_graph* g, int rid) {
  const Resource* r = res_of(g, rid);
  if (!r) return -1;
  if (r->kind == RES_VIEW) r = res_of(g, r->parent);
  return r && r->kind == RES_TRANSIENT ? r->transient_index : -1;
}

static int kind_of_resource(const mtl_graph*, int) { return MTL_KIND_BUFFER; }

// Pass ids in declaration order: the shared update pass is declared first
// whenever it exists (updates_pass!, ext/MantleLavaExt.jl:785-792).
static std::vector<int> declaration_order(const mtl_graph* g) {
  std::vector<int> d;
  if (g->update_pass >= 0) d.push_back(g->update_pass);
  for (int i = 0; i < (int)g->passes.size(); ++i)
    if (i != g->update_pass) d.push_back(i);
  return d;
}

static void add_unique(std::vector<int>& v, int x) {
  if (std::find(v.begin(), v.end(), x) == v.end()) v.push_back(x);
}

// ── elementwise fusion ──────────────────────────────────────────────────────
struct Step {
  std::vector<int> members;  // pass ids, in execution order
  std::vector<std::pair<int, uint32_t>> usages;
};

// A pass that can join a fused run: one elementwise dispatch over a 1-D range,
// every argument a whole declared resource of the graph, no scratch.
static bool fusable(const mtl_graph* g, const Pass& p) {
  if (p.kind != MTL_PASS_COMPUTE || p.dispatches.size() != 1) return false;
  const Dispatch& d = p.dispatches[0];
  const KernelDesc* kd = kernel_desc(d.kernel);
  if (!kd || !kd->elementwise || !kd->ew_emit || d.ndim != 1 || d.workspace_rid) return false;
  for (const mtl_arg& a : d.args)
    if (a.kind == MTL_ARG_PTR) return false;
  for (auto& u : p.usages) {
    const Resource* r = res_of(g, u.first);
    if (!r || r->kind == RES_VIEW || base_of(u.second) != MTL_U_STORAGE) return false;
  }
  return true;
}

bool mtl_pass_compilable(const mtl_graph* g, int pid) {
  return pid >= 0 && pid < (int)g->passes.size() && fusable(g, g->passes[pid]);
}

// The micro-op program of a run, with resource ids standing in for pointers:
// it fails when the run exceeds what one fused kernel can hold.
static bool program_fits(const mtl_graph* g, const std::vector<int>& run) {
  std::vector<EwMember> ms;
  for (int pid : run) {
    const Dispatch& d = g->passes[pid].dispatches[0];
    EwMember m;
    m.kd = kernel_desc(d.kernel);
    m.la.nd[0] = d.nd[0];
    for (const mtl_arg& x : d.args) {
      Arg a;
      a.kind = x.kind == MTL_ARG_RESOURCE ? MTL_ARG_PTR : x.kind;
      a.ptr = x.kind == MTL_ARG_RESOURCE ? (uint64_t)x.rid : 0;
      a.rid = x.kind == MTL_ARG_RESOURCE ? x.rid : 0;
      a.f32 = x.v.f32;
      a.i32 = x.v.i32;
      a.i64 = x.v.i64;
      a.f64 = x.v.f64;
      m.la.a.push_back(a);
    }
    ms.push_back(m);
  }
  EwProgram prog;
  std::string saved = mtl_last_error();
  bool ok = ew_build_program(ms, {}, prog) == MTL_OK && ew_program_fits(prog);
  set_error("%s", saved.c_str());
  return ok;
}

void fuse_steps(mtl_graph* g, const std::vector<int>& decl, const std::vector<int>& order, bool fuse,
                std::vector<Step>& steps, std::vector<int64_t>& elided_at) {
  steps.clear();
  const int n = (int)order.size();
  std::vector<std::vector<int>> runs;
  for (int p = 0; p < n; ++p) {
    int pid = decl[order[p]];
    const Pass& ps = g->passes[pid];
    bool joined = false;
    if (fuse && fusable(g, ps) && !runs.empty() && runs.back().size() >= 1) {
      std::vector<int>& r = runs.back();
      const Pass& head = g->passes[r[0]];
      if (fusable(g, head) && head.dispatches[0].nd[0] == ps.dispatches[0].nd[0]) {
        r.push_back(pid);
        if (program_fits(g, r))
          joined = true;
        else
          r.pop_back();
      }
    }
    if (!joined) runs.push_back({pid});
  }
  // A transient is elided when every pass that touches it is in one fused run
  // and the first of them writes it without reading it: its value then lives in
  // registers only.
  auto& ts = g->transients;
  std::vector<int> step_of(g->passes.size(), -1);
  for (int k = 0; k < (int)runs.size(); ++k)
    for (int pid : runs[k]) step_of[pid] = k;
  std::vector<int> owner(ts.size(), -2);  // -2 untouched, -1 not elidable, else the run
  for (int k = 0; k < (int)runs.size(); ++k)
    for (int pid : runs[k])
      for (auto& u : g->passes[pid].usages) {
        int ti = transient_of(g, u.first);
        if (ti < 0) continue;
        const Resource* r = res_of(g, u.first);
        if (runs[k].size() < 2 || r->kind == RES_VIEW || g->res[ts[ti].rid - 1].internal) {
          owner[ti] = -1;
        } else if (owner[ti] == -2) {
          owner[ti] = usage_writes(u.second) && !usage_reads(u.second) ? k : -1;
        } else if (owner[ti] != k) {
          owner[ti] = -1;
        }
      }
  elided_at.assign(ts.size(), 0);
  for (int k = 0; k < (int)runs.size(); ++k) {
    Step st;
    st.members = runs[k];
    if (runs[k].size() == 1) {
      st.usages = g->passes[runs[k][0]].usages;
    } else {
      // Merged usages: read if the run reads the value from before it, write if
      // the run writes it.
      std::vector<int> rids;
      std::map<int, uint32_t> flags;
      std::set<int> written;
      for (int pid : runs[k])
        for (auto& u : g->passes[pid].usages) {
          int ti = transient_of(g, u.first);
          if (ti >= 0 && owner[ti] == k) continue;
          if (!flags.count(u.first)) rids.push_back(u.first);
          uint32_t& f = flags[u.first];
          f |= MTL_U_STORAGE;
          if (usage_reads(u.second) && !written.count(u.first)) f |= MTL_U_READ;
          if (usage_writes(u.second)) {
            f |= MTL_U_WRITE;
            written.insert(u.first);
          }
        }
      for (int rid : rids) st.usages.push_back({rid, flags[rid]});
    }
    steps.push_back(st);
  }
  for (size_t ti = 0; ti < ts.size(); ++ti)
    if (owner[ti] >= 0) elided_at[ti] = owner[ti] + 1;
  (void)step_of;
}

// ── compile phases ──────────────────────────────────────────────────────────
mtl_status analyze(mtl_graph* g, const CompileOpts& o, Analysis& a) {
  std::vector<int> decl = declaration_order(g);
  const int n = (int)decl.size();
  auto P = [&](int k) -> const Pass& { return g->passes[decl[k]]; };

  // Dag, ext/MantleLavaExt.jl:1353-1368: j depends on i < j when some pair of
  // their usages overlaps and at least one of the two writes.
  std::vector<std::vector<int>> deps(n);
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < j; ++i) {
      bool shared = false;
      for (auto& [idj, Uj] : P(j).usages) {
        for (auto& [idi, Ui] : P(i).usages) {
          if (!overlapping(g, idi, idj)) continue;
          if (!(usage_writes(Ui) || usage_writes(Uj))) continue;
          shared = true;
          break;
        }
        if (shared) break;
      }
      if (shared) deps[j].push_back(i);
    }

  // Schedule, ext/MantleLavaExt.jl:1385-1466: greedy list scheduling under a
  // packed score; objectives sit in disjoint bit ranges (src/phases.jl:55-58).
  std::vector<int> order;
  if (n > 0) {
    const int64_t SCORE_MAX = 0x1fff;
    std::vector<int> remaining(n);
    std::vector<std::vector<int>> dependents(n);
    for (int j = 0; j < n; ++j) {
      remaining[j] = (int)deps[j].size();
      for (int i : deps[j]) dependents[i].push_back(j);
    }
    std::vector<std::vector<int>> ids(n);
    for (int k = 0; k < n; ++k)
      for (auto& u : P(k).usages) add_unique(ids[k], u.first);
    std::map<int, int> touches, seen;
    for (int k = 0; k < n; ++k)
      for (int id : ids[k]) touches[id]++;
    auto bytesof = [&](int id) -> int64_t {
      const Resource* r = res_of(g, id);
      if (!r || r->kind != RES_TRANSIENT) return 0;
      return (int64_t)g->transients[r->transient_index].bytes;
    };
    int64_t maxalloc = 0;
    for (int k = 0; k < n; ++k) {
      int64_t s = 0;
      for (int id : ids[k]) s += bytesof(id);
      maxalloc = std::max(maxalloc, s);
    }
    maxalloc = std::max<int64_t>(1, maxalloc);
    int mshift = o.policy == MTL_POLICY_COMPACT ? 16 : 0;
    int oshift = o.policy == MTL_POLICY_COMPACT ? 0 : 16;
    std::vector<int> ready;
    for (int k = 0; k < n; ++k)
      if (remaining[k] == 0) ready.push_back(k);
    while (!ready.empty()) {
      int best = -1;
      int64_t bestscore = -1;
      for (int r = 0; r < (int)ready.size(); ++r) {
        int i = ready[r];
        int64_t alloc = 0, freed = 0;
        for (int id : ids[i]) {
          int64_t b = bytesof(id);
          if (b == 0) continue;
          int s = seen.count(id) ? seen[id] : 0;
          if (s == 0) alloc += b;
          if (s + 1 == touches[id]) freed += b;
        }
        int64_t m1 = std::clamp<int64_t>((SCORE_MAX * (maxalloc - alloc)) / maxalloc, 0, SCORE_MAX);
        int64_t m2 = std::clamp<int64_t>((SCORE_MAX * freed) / maxalloc, 0, SCORE_MAX);
        int64_t mem = m1 + m2;
        // ord = clamp(n - i, 0, 0xffff) with the reference's 1-based i.
        int64_t ord = std::clamp<int64_t>(n - (i + 1), 0, 0xffff);
        int64_t score = (mem << mshift) | (ord << oshift);
        if (score > bestscore) {
          best = r;
          bestscore = score;
        }
      }
      int i = ready[best];
      ready.erase(ready.begin() + best);
      order.push_back(i);
      for (int id : ids[i]) seen[id]++;
      for (int j : dependents[i])
        if (--remaining[j] == 0) ready.push_back(j);
    }
    if ((int)order.size() != n)
      return fail(MTL_ERR_ARGUMENT, "scheduling left %d passes unreachable: cycle in the DAG",
                  n - (int)order.size());
  }
  // order[] holds declaration positions; positions in the schedule are 1-based
  // below, as in the reference.
  // Steps: every scheduled pass on its own or, when fusion is asked for, runs of
  // consecutive elementwise passes merged into one kernel (fuse_steps). The
  // phases below work on steps, so a fused run is one position: its resources
  // are live together and the placer never gives two of them the same bytes.
  auto& ts = g->transients;
  std::vector<Step> steps;
  std::vector<int64_t> elided_at(ts.size(), 0);  // fused position of an elided transient
  fuse_steps(g, decl, order, o.fuse, steps, elided_at);
  const int ns = (int)steps.size();

  // Liveness, ext/MantleLavaExt.jl:1478-1507: the interval of every transient
  // is recomputed from the scheduled order. A pass that names only a slice of a
  // transient counts as touching it (the reference keys this lookup by the
  // parent's id alone, so a slice-only use would not extend the interval and
  // the placer could hand those bytes to another transient live at that pass).
  for (size_t i = 0; i < ts.size(); ++i) {
    ts[i].first = elided_at[i] ? elided_at[i] : INT64_MAX;
    ts[i].last = elided_at[i];
  }
  for (int p = 0; p < ns; ++p)
    for (auto& u : steps[p].usages) {
      int ti = transient_of(g, u.first);
      if (ti < 0) continue;
      ts[ti].first = std::min<int64_t>(ts[ti].first, p + 1);
      ts[ti].last = std::max<int64_t>(ts[ti].last, p + 1);
    }
  int64_t lastpass = 0;
  for (size_t i = 0; i < ts.size(); ++i) {
    if (ts[i].last == 0) {
      const Resource* r = res_of(g, ts[i].rid);
      return fail(MTL_ERR_ARGUMENT,
                  "transient %zu (Transient.Buffer(%u-byte elements, %llu)) is never used by any "
                  "pass. A transient's interval is derived from use, so one that nothing reads or "
                  "writes has nothing to place. Give it to a pass, or drop the declaration.",
                  i + 1, r->elem_bytes, (unsigned long long)r->elems);
    }
    lastpass = std::max(lastpass, ts[i].last + 1);
  }
  a.items.clear();
  for (size_t i = 0; i < ts.size(); ++i) {
    Item it;
    it.id = std::to_string(i + 1);
    it.lower = o.alias ? ts[i].first : 0;
    it.upper = o.alias ? ts[i].last + 1 : lastpass;
    it.size = elided_at[i] ? 0 : (int64_t)ts[i].bytes;  // an elided transient takes no bytes
    it.alignment = ts[i].alignment;
    a.items.push_back(it);
  }

  // Place, ext/MantleLavaExt.jl:1549-1568: one arena (buffers only).
  a.offsets.assign(ts.size(), 0);
  a.peak = 0;
  a.naive = 0;
  for (auto& t : ts) a.naive += (int64_t)t.bytes;
  if (!ts.empty()) {
    Placement pl;
    mtl_status st = place(a.items, MTL_LOWEST_FIT, pl);
    if (st) return st;
    a.offsets = pl.offsets;
    a.peak = pl.height;
  }

  // Aliasing, ext/MantleLavaExt.jl:1582-1593.
  a.alias_begins.clear();
  for (size_t i = 0; i < ts.size(); ++i)
    for (size_t j = 0; j < ts.size(); ++j) {
      if (i == j) continue;
      const Transient &y = ts[i], &x = ts[j];
      if (!(x.last < y.first)) continue;
      if (a.offsets[i] < a.offsets[j] + a.items[j].size && a.offsets[j] < a.offsets[i] + a.items[i].size)
        a.alias_begins[(int)y.first].push_back({(int)i, (int)j});
    }

  // Barriers, ext/MantleLavaExt.jl:1650-1822. Atomic segments first: every
  // declared range cuts its buffer, and a usage stands for the segments its own
  // range covers (a whole-resource usage for all of them).
  std::map<int, std::vector<int>> slices;  // sliceindex, :1621-1627
  std::map<int, std::vector<std::pair<int64_t, int64_t>>> byparent;
  std::vector<std::tuple<int, int64_t, int64_t, int>> declared;
  for (auto& [key, vid] : g->views) declared.push_back({key.first, key.second.first, key.second.second, vid});
  for (auto& [pid, f, l, vid] : declared) {
    slices[pid].push_back(vid);
    byparent[pid].push_back({f, l});
  }
  a.segments.clear();
  for (auto& [pid, ranges] : byparent) {
    int64_t nel = (int64_t)res_of(g, pid)->elems;
    std::vector<int64_t> cuts = {1, nel + 1};
    for (auto& r : ranges) {
      cuts.push_back(r.first);
      cuts.push_back(r.second + 1);
    }
    std::sort(cuts.begin(), cuts.end());
    cuts.erase(std::unique(cuts.begin(), cuts.end()), cuts.end());
    std::vector<std::pair<int64_t, int64_t>> spans;
    for (size_t k = 0; k + 1 < cuts.size(); ++k)
      if (cuts[k + 1] - 1 >= cuts[k]) spans.push_back({cuts[k], cuts[k + 1] - 1});
    std::vector<int> sids;
    for (auto& s : spans) sids.push_back(intern_view(g, pid, s.first, s.second));
    a.segments[pid] = sids;
    for (auto& r : ranges) {
      int sid = g->views[{pid, r}];
      std::vector<int> cover;
      for (size_t k = 0; k < spans.size(); ++k)
        if (spans[k].first >= r.first && spans[k].second <= r.second) cover.push_back(sids[k]);
      a.segments[sid] = cover;
    }
  }
  auto segments_of = [&](int id) -> std::vector<int> {
    auto it = a.segments.find(id);
    if (it != a.segments.end()) return it->second;
    return {id};
  };

  // A plan is replayed: each segment's state at the start of a replay is its
  // last usage in the schedule (ext/MantleLavaExt.jl:1694-1708).
  std::map<int, uint32_t> final_usage;
  for (int p = 0; p < ns; ++p)
    for (auto& [id, U] : steps[p].usages)
      for (int sid : segments_of(id)) final_usage[sid] = U;

  std::map<int, ResourceState> states;
  auto state = [&](int sid) -> ResourceState& {
    auto it = states.find(sid);
    if (it != states.end()) return it->second;
    ResourceState st;
    auto f = final_usage.find(sid);
    if (f != final_usage.end()) st.current = f->second;
    return states.emplace(sid, st).first->second;
  };

  // Positions (1-based) at which each transient was touched, and per segment
  // the accesses of one replay in scheduled order, for the edge lowering.
  std::vector<std::vector<int>> touched_at(ts.size());
  std::map<int, std::vector<std::pair<int, uint32_t>>> accesses;

  a.prepass.assign(ns, {});
  a.edges.assign(ns, {});
  a.transitions.clear();
  for (int p = 0; p < ns; ++p) {
    const Step& ps = steps[p];
    const int pos = p + 1;
    std::vector<Transition> pre;
    std::vector<int>& edges = a.edges[p];
    for (auto& [id, U] : ps.usages) {
      for (int sid : segments_of(id)) {
        transition_step(pre, MTL_BACKEND_CUDA, kind_of_resource(g, sid), sid, state(sid), U);
        // Lowering: a CUDA graph edge is a dependency between two launches and
        // nothing else, so unlike a pipeline barrier it does not order the
        // passes on either side of it against each other. Each conflicting pair
        // is therefore ordered directly: the same segment, at least one side
        // writes, and not both unordered. Scanning back, an ordered write ends
        // the scan — everything before it is already ordered before it.
        auto& acc = accesses[sid];
        for (int k = (int)acc.size() - 1; k >= 0; --k) {
          auto [q, V] = acc[k];
          bool conflict = (usage_writes(V) || usage_writes(U)) && !(is_unordered(V) && is_unordered(U));
          if (conflict && q != pos) add_unique(edges, q);
          if (usage_writes(V) && !is_unordered(V) && q != pos) break;
        }
        acc.push_back({pos, U});
      }
      int ti = transient_of(g, id);
      if (ti >= 0) add_unique(touched_at[ti], pos);
    }
    std::vector<Transition> needed = pre;

    // Handover where bytes change hands (:1793-1806): the new tenant's first
    // usage waits on what every vacating transient was last doing.
    auto hit = a.alias_begins.find(pos);
    if (hit != a.alias_begins.end()) {
      std::vector<int> news;
      for (auto& h : hit->second) add_unique(news, h.first);
      for (int newi : news) {
        int nrid = ts[newi].rid;
        uint32_t to = 0;
        for (auto& [rid, U] : ps.usages)
          if (overlapping(g, rid, nrid)) {
            to = U;
            break;
          }
        if (to == 0) continue;
        std::vector<uint32_t> waits;
        for (auto& [ni, oi] : hit->second) {
          if (ni != newi) continue;
          int orid = ts[oi].rid;
          std::vector<int> keys = {orid};
          for (int s : slices[orid]) keys.push_back(s);
          for (int s : segments_of(orid)) keys.push_back(s);
          for (int k : keys) {
            auto sit = states.find(k);
            if (sit == states.end() || sit->second.current == 0) continue;
            uint32_t c = sit->second.current;
            if (std::find(waits.begin(), waits.end(), c) == waits.end()) waits.push_back(c);
          }
        }
        if (waits.empty()) continue;
        Transition h;
        h.resource = 0;
        h.from = waits[0];
        h.waits = waits;
        h.to = to;
        needed.push_back(h);
      }
    }
    a.prepass[p] = needed;
    a.transitions.insert(a.transitions.end(), pre.begin(), pre.end());
  }

  // Aliased transients: every pass touching the vacating one is ordered before
  // every pass touching the new tenant (the reduction below keeps only the
  // edges into the tenant's first passes).
  for (auto& [first, pairs] : a.alias_begins)
    for (auto& [yi, xi] : pairs)
      for (int qy : touched_at[yi])
        for (int qx : touched_at[xi])
          if (qx < qy) add_unique(a.edges[qy - 1], qx);

  // Transitive reduction: edges only point forward in the schedule, so walking
  // each pass's predecessors from the latest down, one that is already an
  // ancestor of a kept predecessor is redundant.
  {
    const int W = (ns + 64) / 64;
    std::vector<std::vector<uint64_t>> reach(ns + 1, std::vector<uint64_t>(W, 0));
    auto has = [&](const std::vector<uint64_t>& b, int q) { return (b[q >> 6] >> (q & 63)) & 1; };
    for (int p = 0; p < ns; ++p) {
      std::vector<int>& e = a.edges[p];
      std::sort(e.begin(), e.end(), std::greater<int>());
      std::vector<uint64_t> covered(W, 0);
      std::vector<int> kept;
      for (int q : e) {
        if (has(covered, q)) continue;
        kept.push_back(q);
        covered[q >> 6] |= uint64_t(1) << (q & 63);
        for (int w = 0; w < W; ++w) covered[w] |= reach[q][w];
      }
      reach[p + 1] = covered;
      std::sort(kept.begin(), kept.end());
      e = kept;
    }
  }

  // Report in pass ids (creation order), not declaration positions: each
  // step by its first pass, and every member of every step.
  a.order.resize(ns);
  a.steps.resize(ns);
  for (int p = 0; p < ns; ++p) {
    a.order[p] = steps[p].members[0];
    a.steps[p] = steps[p].members;
  }
  a.elided.clear();
  for (size_t i = 0; i < ts.size(); ++i)
    if (elided_at[i]) a.elided.push_back(ts[i].rid);
  a.deps.assign(g->passes.size(), {});
  for (int j = 0; j < n; ++j)
    for (int i : deps[j]) a.deps[decl[j]].push_back(decl[i]);
  return MTL_OK;
}

}  // namespace mtl

using namespace mtl;

// ── C ABI: vocabulary, transitions, placement ───────────────────────────────
extern "C" {

const char* mtl_last_error(void) { return g_last_error.c_str(); }
int32_t mtl_abi_version(void) { return MTL_ABI_VERSION; }

mtl_status mtl_inject_failure(const char* entry_point, int32_t count) {
  if (!entry_point) return fail(MTL_ERR_ARGUMENT, "mtl_inject_failure: entry point is NULL");
  std::lock_guard<std::mutex> lk(g_inject_mu);
  if (count <= 0)
    g_inject.erase(entry_point);
  else
    g_inject[entry_point] = count;
  return MTL_OK;
}

int32_t mtl_usage_reads(uint32_t u) { return usage_reads(u); }
int32_t mtl_usage_writes(uint32_t u) { return usage_writes(u); }
int32_t mtl_usage_discards(uint32_t u) { return usage_discards(u); }

int32_t mtl_needs_transition(int32_t backend, int32_t kind, uint32_t before, uint32_t after) {
  return needs_transition(backend, kind, before, after);
}

static mtl_status copy_transitions(const std::vector<Transition>& ts, mtl_transition* out,
                                   int32_t cap, int32_t* n) {
  if (n) *n = (int32_t)ts.size();
  for (int32_t i = 0; i < (int32_t)ts.size() && i < cap; ++i) {
    const Transition& t = ts[i];
    if (t.waits.size() > MTL_MAX_WAITS)
      return fail(MTL_ERR_UNSUPPORTED, "transition waits on %zu usages (max %d)", t.waits.size(),
                  MTL_MAX_WAITS);
    out[i].resource = t.resource;
    out[i].from = t.from;
    out[i].to = t.to;
    out[i].nwaits = (int32_t)t.waits.size();
    for (size_t k = 0; k < t.waits.size(); ++k) out[i].waits[k] = t.waits[k];
  }
  return MTL_OK;
}

mtl_status mtl_transitions(int32_t backend, int32_t kind, const uint32_t* usages, int32_t nusages,
                           uint32_t initial, mtl_transition* out, int32_t cap, int32_t* n) {
  if (nusages < 0 || (nusages > 0 && !usages))
    return fail(MTL_ERR_ARGUMENT, "mtl_transitions: bad usage list");
  for (int32_t i = 0; i < nusages; ++i)
    if (!usage_valid(usages[i])) return fail(MTL_ERR_ARGUMENT, "usage code 0x%x is not valid", usages[i]);
  ResourceState st;
  st.current = initial;
  std::vector<Transition> ts;
  for (int32_t i = 0; i < nusages; ++i) transition_step(ts, backend, kind, 1, st, usages[i]);
  return copy_transitions(ts, out, cap, n);
}

static mtl_status items_from(const mtl_item* items, int32_t n, std::vector<Item>& v) {
  if (n < 0 || (n > 0 && !items)) return fail(MTL_ERR_ARGUMENT, "bad item list");
  v.resize(n);
  for (int32_t i = 0; i < n; ++i) {
    const mtl_item& s = items[i];
    Item& it = v[i];
    it.id = s.id ? s.id : std::to_string(i + 1);
    it.lower = s.lower;
    it.upper = s.upper;
    it.size = s.size;
    it.alignment = s.alignment < 1 ? 1 : s.alignment;
    it.offset = s.offset;
    for (int32_t k = 0; k < s.ngaps; ++k) {
      Gap gp;
      gp.lower = s.gaps[k].lower;
      gp.upper = s.gaps[k].upper;
      gp.has_window = s.gaps[k].window_lower >= 0;
      gp.wlo = s.gaps[k].window_lower;
      gp.whi = s.gaps[k].window_upper;
      it.gaps.push_back(gp);
    }
  }
  return MTL_OK;
}

mtl_status mtl_place(const mtl_item* items, int32_t n, int32_t strategy, int64_t* offsets,
                     int64_t* height) {
  std::vector<Item> v;
  mtl_status st = items_from(items, n, v);
  if (st) return st;
  Placement pl;
  st = place(v, strategy, pl);
  if (st) return st;
  for (int32_t i = 0; i < n; ++i) offsets[i] = pl.offsets[i];
  if (height) *height = pl.height;
  return MTL_OK;
}

mtl_status mtl_maxload(const mtl_item* items, int32_t n, int64_t* out) {
  std::vector<Item> v;
  mtl_status st = items_from(items, n, v);
  if (st) return st;
  *out = maxload(v);
  return MTL_OK;
}

// ── C ABI: graph recording ──────────────────────────────────────────────────
mtl_status mtl_graph_create(mtl_device* dev, mtl_graph** out) {
  if (!out) return fail(MTL_ERR_ARGUMENT, "mtl_graph_create: out is NULL");
  if (mtl_status s = injected("mtl_graph_create")) return s;
  *out = new mtl_graph();
  (*out)->dev = dev;
  if (dev) retain_device(dev);
  return MTL_OK;
}

mtl_status mtl_graph_release(mtl_graph* g) {
  if (g) release_graph(g);
  return MTL_OK;
}

mtl_status mtl_graph_persistent(mtl_graph* g, mtl_buffer* buf, uint64_t elems, uint32_t elem_bytes,
                                int32_t* rid) {
  if (!g || !rid) return fail(MTL_ERR_ARGUMENT, "mtl_graph_persistent: NULL argument");
  if (elem_bytes == 0) return fail(MTL_ERR_ARGUMENT, "mtl_graph_persistent: zero-byte elements");
  if (buf) {
    auto it = g->persistent_ids.find(buf);
    if (it != g->persistent_ids.end()) {
      *rid = it->second;
      return MTL_OK;
    }
  }
  Resource r;
  r.kind = RES_PERSISTENT;
  r.elems = elems;
  r.elem_bytes = elem_bytes;
  r.buf = buf;
  g->res.push_back(r);
  *rid = (int32_t)g->res.size();
  if (buf) {
    g->persistent_ids[buf] = *rid;
    retain_buffer(buf);
  }
  return MTL_OK;
}

static int new_transient(mtl_graph* g, uint64_t elems, uint32_t elem_bytes, bool internal) {
  Resource r;
  r.kind = RES_TRANSIENT;
  r.elems = elems;
  r.elem_bytes = elem_bytes;
  r.transient_index = (int)g->transients.size();
  r.internal = internal;
  g->res.push_back(r);
  int rid = (int)g->res.size();
  Transient t;
  t.rid = rid;
  t.bytes = elems * elem_bytes;
  g->transients.push_back(t);
  return rid;
}

mtl_status mtl_graph_transient(mtl_graph* g, uint64_t elems, uint32_t elem_bytes, int32_t* rid) {
  if (!g || !rid) return fail(MTL_ERR_ARGUMENT, "mtl_graph_transient: NULL argument");
  if (elem_bytes == 0) return fail(MTL_ERR_ARGUMENT, "mtl_graph_transient: zero-byte elements");
  *rid = new_transient(g, elems, elem_bytes, false);
  return MTL_OK;
}

mtl_status mtl_graph_pass(mtl_graph* g, const char* name, int32_t kind, int32_t* pass) {
  if (!g || !pass) return fail(MTL_ERR_ARGUMENT, "mtl_graph_pass: NULL argument");
  if (kind != MTL_PASS_COMPUTE && kind != MTL_PASS_CUSTOM)
    return fail(MTL_ERR_ARGUMENT, "mtl_graph_pass: kind must be compute or custom");
  Pass p;
  p.name = name ? name : "";
  p.kind = kind;
  g->passes.push_back(p);
  *pass = (int32_t)g->passes.size() - 1;
  return MTL_OK;
}

static bool valid_pass(mtl_graph* g, int32_t pass) { return pass >= 0 && pass < (int)g->passes.size(); }

mtl_status mtl_graph_use(mtl_graph* g, int32_t pass, int32_t rid, uint32_t usage, int64_t first,
                         int64_t last, int32_t* out_rid) {
  if (!g) return fail(MTL_ERR_ARGUMENT, "use(): graph is NULL");
  if (!valid_pass(g, pass)) return fail(MTL_ERR_ARGUMENT, "use(): no pass %d", pass);
  const Resource* r = res_of(g, rid);
  if (!r || r->kind == RES_VIEW) return fail(MTL_ERR_ARGUMENT, "use(): no resource %d", rid);
  if (base_of(usage) == MTL_U_STORAGE && (usage & (MTL_U_READ | MTL_U_WRITE)) == 0)
    return fail(MTL_ERR_ARGUMENT, "use() needs read, write, or both");
  if (!usage_valid(usage)) return fail(MTL_ERR_ARGUMENT, "use(): usage code 0x%x is not valid", usage);
  int id = rid;
  if (first != 0) {
    int64_t nel = (int64_t)r->elems;
    if (!(first >= 1 && last <= nel && last >= first - 1))
      return fail(MTL_ERR_ARGUMENT, "use(): range %lld:%lld is outside the buffer's 1:%lld.",
                  (long long)first, (long long)last, (long long)nel);
    id = intern_view(g, rid, first, last);
  }
  g->passes[pass].usages.push_back({id, usage});
  if (out_rid) *out_rid = id;
  return MTL_OK;
}

mtl_status mtl_graph_dispatch(mtl_graph* g, int32_t pass, int32_t kernel, const mtl_arg* args,
                              int32_t nargs, const int64_t* ndrange, int32_t ndim,
                              const int32_t* group) {
  if (!g) return fail(MTL_ERR_ARGUMENT, "dispatch!: graph is NULL");
  if (!valid_pass(g, pass)) return fail(MTL_ERR_ARGUMENT, "dispatch!: no pass %d", pass);
  Pass& p = g->passes[pass];
  if (p.kind != MTL_PASS_COMPUTE) return fail(MTL_ERR_ARGUMENT, "dispatch!: pass \"%s\" is not a compute pass", p.name.c_str());
  const KernelDesc* kd = kernel_desc(kernel);
  if (!kd) return fail(MTL_ERR_ARGUMENT, "dispatch!: unknown kernel %d", kernel);
  int want = (int)strlen(kd->sig);
  if (nargs != want)
    return fail(MTL_ERR_ARGUMENT, "dispatch!: kernel %s takes %d arguments (%s), got %d", kd->name,
                want, kd->sig, nargs);
  if (ndim < 1 || ndim > 3 || !ndrange) return fail(MTL_ERR_ARGUMENT, "dispatch!: ndrange must have 1-3 dimensions");
  for (int i = 0; i < ndim; ++i)
    if (ndrange[i] < 0) return fail(MTL_ERR_ARGUMENT, "dispatch!: negative ndrange");
  for (int i = 0; i < nargs; ++i) {
    char c = kd->sig[i];
    int k = args[i].kind;
    bool ok;
    switch (c) {
      case 'B': ok = k == MTL_ARG_RESOURCE || k == MTL_ARG_PTR; break;
      case 'b': ok = k == MTL_ARG_RESOURCE || k == MTL_ARG_PTR || k == MTL_ARG_NULL; break;
      case 'f': ok = k == MTL_ARG_F32; break;
      case 'i': ok = k == MTL_ARG_I32; break;
      case 'I': ok = k == MTL_ARG_I64; break;
      case 'd': ok = k == MTL_ARG_F64; break;
      default: ok = false;
    }
    if (!ok)
      return fail(MTL_ERR_ARGUMENT, "dispatch!: kernel %s argument %d has the wrong kind (%s)",
                  kd->name, i + 1, kd->sig);
    if (k == MTL_ARG_RESOURCE && !res_of(g, args[i].rid))
      return fail(MTL_ERR_ARGUMENT, "dispatch!: kernel %s argument %d names no resource", kd->name, i + 1);
  }
  Dispatch d;
  d.kernel = kernel;
  d.args.assign(args, args + nargs);
  d.ndim = ndim;
  for (int i = 0; i < ndim; ++i) d.nd[i] = ndrange[i];
  if (group)
    for (int i = 0; i < ndim; ++i) d.group[i] = group[i];
  // A kernel that needs scratch gets it as a transient of its own, written by
  // this pass only, so the placer may share its bytes with anything whose
  // lifetime is disjoint.
  if (kd->workspace) {
    LaunchArgs la;
    la.ndim = ndim;
    for (int i = 0; i < ndim; ++i) la.nd[i] = ndrange[i];
    for (int i = 0; i < nargs; ++i) {
      Arg a;
      a.kind = args[i].kind == MTL_ARG_RESOURCE ? MTL_ARG_PTR : args[i].kind;
      a.ptr = args[i].kind == MTL_ARG_PTR ? args[i].v.ptr : (args[i].kind == MTL_ARG_RESOURCE ? 1 : 0);
      a.f32 = args[i].v.f32;
      a.i32 = args[i].v.i32;
      a.i64 = args[i].v.i64;
      a.f64 = args[i].v.f64;
      la.a.push_back(a);
    }
    la.sm_count = device_sm_count(g->dev);
    la.device = device_ordinal(g->dev);
    uint64_t bytes = kd->workspace(la);
    if (bytes > 0) {
      d.workspace_rid = new_transient(g, (bytes + 255) / 256, 256, true);
      p.usages.push_back({d.workspace_rid, MTL_U_STORAGE | MTL_U_READ | MTL_U_WRITE});
    }
  }
  p.dispatches.push_back(d);
  return MTL_OK;
}

mtl_status mtl_graph_custom(mtl_graph* g, int32_t pass, mtl_custom_fn fn, void* user) {
  if (!g) return fail(MTL_ERR_ARGUMENT, "custom!: graph is NULL");
  if (!valid_pass(g, pass)) return fail(MTL_ERR_ARGUMENT, "custom!: no pass %d", pass);
  Pass& p = g->passes[pass];
  if (p.kind != MTL_PASS_CUSTOM) return fail(MTL_ERR_ARGUMENT, "custom!: pass \"%s\" is not a custom pass", p.name.c_str());
  if (!fn)
    return fail(MTL_ERR_ARGUMENT,
                "custom!: the block has to return a zero-argument callable — it is what runs at "
                "record time. Declare the uses, then return the work.");
  p.custom_fn = fn;
  p.custom_user = user;
  return MTL_OK;
}

mtl_status mtl_graph_copy(mtl_graph* g, const char* name, int32_t dst_rid, int32_t src_rid,
                          int32_t* pass) {
  if (!g || !pass) return fail(MTL_ERR_ARGUMENT, "copy!: NULL argument");
  const Resource* d = res_of(g, dst_rid);
  const Resource* s = res_of(g, src_rid);
  if (!d || !s || d->kind == RES_VIEW || s->kind == RES_VIEW)
    return fail(MTL_ERR_ARGUMENT, "copy!: source and destination must be buffers of this graph");
  if (d->elems * d->elem_bytes < s->elems * s->elem_bytes)
    return fail(MTL_ERR_ARGUMENT, "copy!: destination (%llu bytes) is smaller than the source (%llu bytes)",
                (unsigned long long)(d->elems * d->elem_bytes), (unsigned long long)(s->elems * s->elem_bytes));
  Pass p;
  p.name = name ? name : "copy";
  p.kind = MTL_PASS_COPY;
  p.copy_src = src_rid;
  p.copy_dst = dst_rid;
  p.usages.push_back({src_rid, MTL_U_COPY_SRC});
  p.usages.push_back({dst_rid, MTL_U_COPY_DST});
  g->passes.push_back(p);
  *pass = (int32_t)g->passes.size() - 1;
  return MTL_OK;
}

mtl_status mtl_graph_update(mtl_graph* g, int32_t rid, int64_t first, int64_t last, int32_t* update) {
  if (!g || !update) return fail(MTL_ERR_ARGUMENT, "Update: NULL argument");
  const Resource* r = res_of(g, rid);
  if (!r || r->kind != RES_PERSISTENT) return fail(MTL_ERR_ARGUMENT, "Update: resource %d is not a persistent buffer", rid);
  if (first != 0 && !(first >= 1 && last <= (int64_t)r->elems && last >= first))
    return fail(MTL_ERR_ARGUMENT, "Update: range %lld:%lld is outside the buffer's 1:%llu.",
                (long long)first, (long long)last, (unsigned long long)r->elems);
  if (g->update_pass < 0) {
    Pass p;
    p.name = "updates";
    p.kind = MTL_PASS_UPDATE;
    g->passes.push_back(p);
    g->update_pass = (int)g->passes.size() - 1;
  }
  Pass& up = g->passes[g->update_pass];
  bool have = false;
  for (auto& u : up.usages) have |= u.first == rid;
  if (!have) up.usages.push_back({rid, MTL_U_COPY_DST});
  UpdateDecl d;
  d.rid = rid;
  d.first = first;
  d.last = last;
  g->updates.push_back(d);
  *update = (int32_t)g->updates.size() - 1;
  return MTL_OK;
}

mtl_status mtl_graph_resource(mtl_graph* g, int32_t rid, int32_t* kind, int32_t* parent,
                              int64_t* first, int64_t* last, uint64_t* elems) {
  if (!g) return fail(MTL_ERR_ARGUMENT, "graph is NULL");
  const Resource* r = res_of(g, rid);
  if (!r) return fail(MTL_ERR_ARGUMENT, "no resource %d", rid);
  if (kind) *kind = r->kind;
  if (parent) *parent = r->parent;
  if (first) *first = r->first;
  if (last) *last = r->last;
  if (elems) *elems = r->elems;
  return MTL_OK;
}

mtl_status mtl_graph_npasses(mtl_graph* g, int32_t* n) {
  if (!g || !n) return fail(MTL_ERR_ARGUMENT, "NULL argument");
  *n = (int32_t)g->passes.size();
  return MTL_OK;
}

mtl_status mtl_graph_pass_name(mtl_graph* g, int32_t pass, const char** name) {
  if (!g || !name || !valid_pass(g, pass)) return fail(MTL_ERR_ARGUMENT, "no pass %d", pass);
  *name = g->passes[pass].name.c_str();
  return MTL_OK;
}

}  // extern "C"

namespace mtl {
static std::mutex g_graph_refs_mu;

void retain_graph(mtl_graph* g) {
  std::lock_guard<std::mutex> lk(g_graph_refs_mu);
  ++g->refs;
}

void release_graph(mtl_graph* g) {
  {
    std::lock_guard<std::mutex> lk(g_graph_refs_mu);
    if (--g->refs > 0) return;
  }
  for (auto& kv : g->persistent_ids) release_buffer(kv.first);
  mtl_device* dev = g->dev;
  delete g;
  if (dev) release_device(dev);
}
}  // namespace mtl
