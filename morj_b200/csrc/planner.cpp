// Host planner for the tree-prefill forward: the radix layout of a request's sequences and the plan of one pass
// (steps, positions, tokens, pool slots, CSR page tables, readout rows). The rules are the reference planner's
// (aleria_judge/lean_core.py:34-231, `Tree`), so the outputs are identical to it: node ids, offsets, step cuts,
// slot numbers and readout rows are the contract between passes of one request and the kernels.
//
// Layout rules (lean_core.py:38-83). Sequences are inserted in order; each shares its longest prefix with the earliest
// earlier sequence that has it; a node whose span straddles the branch point is split, the tail becoming a new node
// that follows it on every path through it. Nodes are then numbered by start depth (ties by creation order) and own
// consecutive tree offsets.
//
// Plan rules (lean_core.py:120-231). A pass over more than `single_max` tokens is cut into steps of `step_tokens`
// over the nodes in depth-first order (image blocks never split and open a new step when they do not fit); image
// blocks lead their step. A segment attends over its path's offsets (the last `window` before its first query for
// sliding layers). Slots come from a liveness allocator: computed tokens take the lowest free slots, then new ones;
// with several steps a slot is freed after the last step that reads its token; pinned offsets are never freed.
#include <algorithm>
#include <array>
#include <cstring>
#include <functional>
#include <new>
#include <queue>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "morj_b200.h"

namespace morj {
int set_error(int code, const char* fmt, ...);

namespace plan {

using ll = long long;

struct Tree {
  std::vector<std::vector<ll>> seqs;
  std::vector<std::array<ll, 3>> nodes;  // owner, start depth, end depth
  std::vector<std::vector<int>> paths;   // per sequence: node ids from the root
  std::vector<ll> offsets;               // n_nodes + 1
  std::vector<std::vector<int>> node_path;  // per node: node ids from the root to it
  ll num_tokens = 0;
};

static ll common_prefix(const std::vector<ll>& a, const std::vector<ll>& b) {
  const size_t n = std::min(a.size(), b.size());
  size_t k = 0;
  while (k < n && a[k] == b[k]) ++k;
  return (ll)k;
}

static void build(Tree& t) {
  std::vector<std::array<ll, 3>> raw;  // creation order
  std::vector<std::vector<int>> members;
  for (size_t b = 0; b < t.seqs.size(); ++b) {
    const std::vector<ll>& seq = t.seqs[b];
    int donor = -1;
    ll shared = 0;
    for (size_t j = 0; j < b; ++j) {
      const ll c = common_prefix(seq, t.seqs[j]);
      if (c > shared) {
        donor = (int)j;
        shared = c;
      }
    }
    std::vector<int> route;
    if (donor >= 0) {
      const std::vector<int> walk = members[donor];
      for (int nid : walk) {
        const ll start = raw[nid][1], end = raw[nid][2];
        if (end <= shared) {
          route.push_back(nid);
          continue;
        }
        if (start < shared) {  // the branch point is inside this node: split off its tail
          raw.push_back({raw[nid][0], shared, end});
          const int tail = (int)raw.size() - 1;
          raw[nid][2] = shared;
          for (std::vector<int>& m : members) {
            auto it = std::find(m.begin(), m.end(), nid);
            if (it != m.end()) m.insert(it + 1, tail);
          }
          route.push_back(nid);
        }
        break;
      }
    }
    if (shared < (ll)seq.size()) {
      raw.push_back({(ll)b, shared, (ll)seq.size()});
      route.push_back((int)raw.size() - 1);
    }
    members.push_back(std::move(route));
  }
  std::vector<int> order(raw.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = (int)i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int c) { return raw[a][1] < raw[c][1]; });
  std::vector<int> new_id(raw.size());
  for (size_t k = 0; k < order.size(); ++k) new_id[order[k]] = (int)k;
  t.nodes.resize(raw.size());
  for (size_t k = 0; k < order.size(); ++k) t.nodes[k] = raw[order[k]];
  t.paths.resize(members.size());
  for (size_t b = 0; b < members.size(); ++b)
    for (int n : members[b]) t.paths[b].push_back(new_id[n]);
  t.offsets.assign(t.nodes.size() + 1, 0);
  for (size_t i = 0; i < t.nodes.size(); ++i) t.offsets[i + 1] = t.offsets[i] + (t.nodes[i][2] - t.nodes[i][1]);
  t.num_tokens = t.offsets.back();
  t.node_path.assign(t.nodes.size(), {});
  std::vector<char> seen(t.nodes.size(), 0);
  for (const std::vector<int>& p : t.paths)
    for (size_t i = 0; i < p.size(); ++i)
      if (!seen[p[i]]) {
        seen[p[i]] = 1;
        t.node_path[p[i]].assign(p.begin(), p.begin() + i + 1);
      }
}

struct Seg {
  int node;
  ll a, b;
};

// Pass plan, serialised as one int64 blob (layout in morj_b200.h, morj_plan_pass).
struct Plan {
  std::vector<ll> blob;
};

static bool readout_slot(const Tree& t, int b, int* node, ll* offset) {
  const ll last = (ll)t.seqs[b].size() - 1;
  for (int nid : t.paths[b]) {
    const ll s = t.nodes[nid][1], e = t.nodes[nid][2];
    if (s <= last && last < e) {
      *node = nid;
      *offset = t.offsets[nid] + last - s;
      return true;
    }
  }
  return false;
}

static std::vector<int> depth_first(const Tree& t, const std::vector<int>& compute) {
  std::unordered_set<int> todo(compute.begin(), compute.end());
  std::unordered_map<int, std::vector<int>> kids;
  for (int n : compute) {
    const std::vector<int>& np = t.node_path[n];
    const int parent = np.size() > 1 ? np[np.size() - 2] : -1;
    kids[todo.count(parent) ? parent : -1].push_back(n);
  }
  std::vector<int> out, stack = kids[-1];
  std::sort(stack.begin(), stack.end(), std::greater<int>());
  while (!stack.empty()) {
    const int n = stack.back();
    stack.pop_back();
    out.push_back(n);
    auto it = kids.find(n);
    if (it != kids.end()) {
      std::vector<int> k = it->second;
      std::sort(k.begin(), k.end(), std::greater<int>());
      stack.insert(stack.end(), k.begin(), k.end());
    }
  }
  return out;
}

static std::vector<std::vector<Seg>> cut(const Tree& t, const std::vector<int>& compute, ll budget,
                                         const std::unordered_set<int>& bidir) {
  std::vector<std::vector<Seg>> steps;
  std::vector<Seg> cur;
  ll room = budget;
  for (int n : compute) {
    ll a = t.nodes[n][1];
    const ll end = t.nodes[n][2];
    const bool whole = bidir.count(n) != 0;
    if (whole && end - a > room && !cur.empty()) {
      steps.push_back(std::move(cur));
      cur.clear();
      room = budget;
    }
    while (a < end) {
      const ll take = whole ? end - a : std::min(end - a, room);
      cur.push_back({n, a, a + take});
      a += take;
      room -= take;
      if (room <= 0) {
        steps.push_back(std::move(cur));
        cur.clear();
        room = budget;
      }
    }
  }
  if (!cur.empty()) steps.push_back(std::move(cur));
  for (std::vector<Seg>& st : steps)  // image blocks lead their step
    std::stable_partition(st.begin(), st.end(), [&](const Seg& s) { return bidir.count(s.node) != 0; });
  return steps;
}

struct Step {
  std::vector<Seg> segs;
  std::vector<ll> own;  // tree offsets computed by the step, in row order
  int n_bidir = 0;
};

// The offsets segment `sg` reads, in depth order: its ancestors' whole ranges, then its own node up to its end;
// `skip` leading entries are left out (the sliding list). f(offset) is called for each.
template <class F>
static void for_path(const Tree& t, const Seg& sg, ll skip, F&& f) {
  const std::vector<int>& np = t.node_path[sg.node];
  for (size_t i = 0; i < np.size(); ++i) {
    const ll lo = t.offsets[np[i]];
    const ll hi = i + 1 < np.size() ? t.offsets[np[i] + 1] : t.offsets[sg.node] + (sg.b - t.nodes[sg.node][1]);
    ll o = lo;
    if (skip > 0) {
      const ll drop = std::min(skip, hi - lo);
      o += drop;
      skip -= drop;
    }
    for (; o < hi; ++o) f(o);
  }
}

// Liveness slot allocator for one kind (lean_core.py:198-222).
static ll allocate(const Tree& t, const std::vector<Step>& steps, std::vector<ll>& last, std::vector<ll>& table,
                   const ll* prealloc, ll n_prealloc, const ll* initial, const ll* pinned, ll n_pinned) {
  const ll nt = t.num_tokens;
  table.assign(nt, -1);
  if (initial) {
    std::copy(initial, initial + nt, table.begin());
  } else {
    for (ll i = 0; i < n_prealloc; ++i) table[prealloc[i]] = i;
  }
  if (pinned)
    for (ll i = 0; i < n_pinned; ++i) last[pinned[i]] = (ll)steps.size();
  std::vector<char> resident(nt, 0);
  ll top = 0;
  for (ll i = 0; i < nt; ++i)
    if (table[i] >= 0) {
      resident[i] = 1;
      top = std::max(top, table[i] + 1);
    }
  std::vector<char> taken(top, 0);
  for (ll i = 0; i < nt; ++i)
    if (resident[i]) taken[table[i]] = 1;
  std::priority_queue<ll, std::vector<ll>, std::greater<ll>> free;  // the lowest free slot first
  for (ll s = 0; s < top; ++s)
    if (!taken[s]) free.push(s);
  const bool multi = steps.size() > 1;
  for (size_t k = 0; k < steps.size(); ++k) {
    const std::vector<ll>& own = steps[k].own;
    const size_t reuse = std::min(free.size(), own.size());
    for (size_t i = 0; i < own.size(); ++i) {
      if (i < reuse) {
        table[own[i]] = free.top();
        free.pop();
      } else {
        table[own[i]] = top + (ll)(i - reuse);
      }
      resident[own[i]] = 1;
    }
    top += (ll)(own.size() - reuse);
    if (multi)
      for (ll i = 0; i < nt; ++i)
        if (resident[i] && last[i] <= (ll)k) {
          resident[i] = 0;
          free.push(table[i]);
        }
  }
  return top;
}

// Plan blobs are built in vectors taken from a small per-thread pool, so their pages stay mapped between plans.
static thread_local std::vector<std::vector<ll>> t_pool;

static std::vector<ll> take_buffer() {
  if (t_pool.empty()) return {};
  std::vector<ll> v = std::move(t_pool.back());
  t_pool.pop_back();
  return v;
}

// Returns MORJ_OK, MORJ_ERR_ARG (a readout token is not computed in the pass) or MORJ_ERR_INTERNAL (a segment
// reads a token without a slot).
static int plan_pass(const Tree& t, std::vector<int> compute, const int* readout_seqs, int n_readout, int window,
                     ll single_max, ll step_tokens, int identity, const ll* prealloc, ll n_prealloc,
                     const ll* const initial[2], const ll* const pinned[2], const ll n_pinned[2],
                     const std::unordered_set<int>& bidir, Plan& out) {
  ll total = 0;
  for (int n : compute) total += t.nodes[n][2] - t.nodes[n][1];
  ll budget = total;
  if (total > single_max) {
    budget = step_tokens;
    compute = depth_first(t, compute);
  }
  const std::vector<std::vector<Seg>> cuts = cut(t, compute, budget, bidir);

  std::unordered_map<ll, std::vector<int>> want;  // tree offset -> readout indices
  for (int i = 0; i < n_readout; ++i) {
    int node;
    ll off;
    if (!readout_slot(t, readout_seqs[i], &node, &off))
      return set_error(MORJ_ERR_ARG, "morj_plan_pass: empty sequence");
    want[off].push_back(i);
  }
  std::vector<std::pair<ll, ll>> readout(n_readout, {-1, -1});
  std::vector<ll> last_read[2] = {std::vector<ll>(t.num_tokens, -1), std::vector<ll>(t.num_tokens, -1)};
  std::vector<Step> steps(cuts.size());
  // sliding lists drop the path entries before depth a - window + 1
  auto sliding_skip = [&](const Seg& sg) { return std::min<ll>(std::max<ll>(0, sg.a - window + 1), sg.b); };
  ll blob_size = 5 + 2 * t.num_tokens + 2 * (ll)n_readout;
  for (size_t k = 0; k < cuts.size(); ++k) {
    Step& st = steps[k];
    st.segs = cuts[k];
    ll kv = 0;
    for (const Seg& sg : st.segs) {
      const ll sn = t.nodes[sg.node][1], base = t.offsets[sg.node];
      for_path(t, sg, 0, [&](ll o) { last_read[0][o] = (ll)k; });
      for_path(t, sg, sliding_skip(sg), [&](ll o) { last_read[1][o] = (ll)k; });
      kv += sg.b + (sg.b - sliding_skip(sg));
      for (ll d = sg.a; d < sg.b; ++d) st.own.push_back(base + d - sn);
      if (bidir.count(sg.node)) ++st.n_bidir;
    }
    for (size_t r = 0; r < st.own.size(); ++r) {
      auto it = want.find(st.own[r]);
      if (it != want.end())
        for (int i : it->second) readout[i] = {(ll)k, (ll)r};
    }
    const ll ns = (ll)st.segs.size(), nr = (ll)st.own.size();
    blob_size += 5 + 3 * ns + 3 * nr + (ns + 1) + 2 * nr + 2 * (ns + 1) + kv;
  }
  for (const auto& r : readout)
    if (r.first < 0) return set_error(MORJ_ERR_ARG, "a readout token is not computed in this pass");

  std::vector<ll> slot_of[2];
  ll cap[2];
  for (int kind = 0; kind < 2; ++kind) {
    if (identity) {
      slot_of[kind].resize(t.num_tokens);
      for (ll i = 0; i < t.num_tokens; ++i) slot_of[kind][i] = i;
      cap[kind] = t.num_tokens;
      continue;
    }
    cap[kind] = allocate(t, steps, last_read[kind], slot_of[kind], prealloc, n_prealloc, initial[kind],
                         pinned[kind], n_pinned[kind]);
  }

  std::vector<ll>& blob = out.blob;
  blob = take_buffer();
  blob.resize(blob_size);
  ll* w = blob.data();
  *w++ = t.num_tokens;
  *w++ = (ll)steps.size();
  *w++ = cap[0];
  *w++ = cap[1];
  *w++ = (ll)n_readout;
  for (int kind = 0; kind < 2; ++kind) w = std::copy(slot_of[kind].begin(), slot_of[kind].end(), w);
  for (const auto& r : readout) {
    *w++ = r.first;
    *w++ = r.second;
  }
  bool holes = false;
  for (const Step& st : steps) {
    ll n_kv[2] = {0, 0};
    for (const Seg& sg : st.segs) {
      n_kv[0] += sg.b;
      n_kv[1] += sg.b - sliding_skip(sg);
    }
    *w++ = (ll)st.segs.size();
    *w++ = (ll)st.own.size();
    *w++ = (ll)st.n_bidir;
    *w++ = n_kv[0];
    *w++ = n_kv[1];
    for (const Seg& sg : st.segs) {
      *w++ = sg.node;
      *w++ = sg.a;
      *w++ = sg.b;
    }
    w = std::copy(st.own.begin(), st.own.end(), w);
    for (const Seg& sg : st.segs)
      for (ll d = sg.a; d < sg.b; ++d) *w++ = d;
    for (const Seg& sg : st.segs) {
      const std::vector<ll>& seq = t.seqs[t.nodes[sg.node][0]];
      w = std::copy(seq.begin() + sg.a, seq.begin() + sg.b, w);
    }
    ll q = 0;
    *w++ = 0;
    for (const Seg& sg : st.segs) *w++ = (q += sg.b - sg.a);
    for (int kind = 0; kind < 2; ++kind)
      for (ll o : st.own) *w++ = slot_of[kind][o];
    for (int kind = 0; kind < 2; ++kind) {
      ll acc = 0;
      *w++ = 0;
      for (const Seg& sg : st.segs) *w++ = (acc += kind ? sg.b - sliding_skip(sg) : sg.b);
      const std::vector<ll>& so = slot_of[kind];
      for (const Seg& sg : st.segs)
        for_path(t, sg, kind ? sliding_skip(sg) : 0, [&](ll o) {
          const ll s = so[o];
          holes |= s < 0;
          *w++ = s;
        });
    }
  }
  if (holes) return set_error(MORJ_ERR_INTERNAL, "a segment reads a token that has no slot");
  return MORJ_OK;
}

}  // namespace plan
}  // namespace morj

using morj::plan::ll;

extern "C" int morj_tree_build(const long long* tokens, const long long* seq_indptr, int n_seqs, void** tree) {
  if (!tree || n_seqs < 0 || (n_seqs > 0 && (!seq_indptr || (!tokens && seq_indptr[n_seqs] > 0))))
    return morj::set_error(MORJ_ERR_ARG, "morj_tree_build: bad arguments");
  auto* t = new (std::nothrow) morj::plan::Tree;
  if (!t) return morj::set_error(MORJ_ERR_OOM, "morj_tree_build: out of host memory");
  t->seqs.resize(n_seqs);
  for (int b = 0; b < n_seqs; ++b) {
    if (seq_indptr[b + 1] < seq_indptr[b]) {
      delete t;
      return morj::set_error(MORJ_ERR_ARG, "morj_tree_build: seq_indptr must not decrease");
    }
    t->seqs[b].assign(tokens + seq_indptr[b], tokens + seq_indptr[b + 1]);
  }
  morj::plan::build(*t);
  *tree = t;
  return MORJ_OK;
}

extern "C" int morj_tree_layout(const void* tree, long long* sizes, long long* nodes, long long* offsets,
                                long long* path_indptr, long long* path_ids, long long* node_path_indptr,
                                long long* node_path_ids) {
  if (!tree || !sizes) return morj::set_error(MORJ_ERR_ARG, "morj_tree_layout: bad arguments");
  const auto& t = *static_cast<const morj::plan::Tree*>(tree);
  ll n_path = 0, n_np = 0;
  for (const auto& p : t.paths) n_path += (ll)p.size();
  for (const auto& p : t.node_path) n_np += (ll)p.size();
  sizes[0] = (ll)t.nodes.size();
  sizes[1] = n_path;
  sizes[2] = n_np;
  if (!nodes) return MORJ_OK;  // sizes only
  for (size_t i = 0; i < t.nodes.size(); ++i)
    for (int j = 0; j < 3; ++j) nodes[3 * i + j] = t.nodes[i][j];
  std::copy(t.offsets.begin(), t.offsets.end(), offsets);
  ll k = 0;
  path_indptr[0] = 0;
  for (size_t b = 0; b < t.paths.size(); ++b) {
    for (int n : t.paths[b]) path_ids[k++] = n;
    path_indptr[b + 1] = k;
  }
  k = 0;
  node_path_indptr[0] = 0;
  for (size_t i = 0; i < t.node_path.size(); ++i) {
    for (int n : t.node_path[i]) node_path_ids[k++] = n;
    node_path_indptr[i + 1] = k;
  }
  return MORJ_OK;
}

extern "C" void morj_tree_free(void* tree) { delete static_cast<morj::plan::Tree*>(tree); }

extern "C" int morj_plan_pass(const void* tree, const long long* compute, int n_compute, const int* readout_seqs,
                              int n_readout, int window, long long single_max, long long step_tokens, int identity,
                              const long long* prealloc, long long n_prealloc, const long long* initial_g,
                              const long long* initial_s, const long long* pinned_g, long long n_pinned_g,
                              const long long* pinned_s, long long n_pinned_s, const long long* bidir, int n_bidir,
                              void** plan) {
  if (!tree || !plan || n_compute < 0 || n_readout < 0 || (n_compute && !compute) || (n_readout && !readout_seqs) ||
      (n_prealloc && !prealloc) || (n_bidir && !bidir) || step_tokens <= 0)
    return morj::set_error(MORJ_ERR_ARG, "morj_plan_pass: bad arguments");
  const auto& t = *static_cast<const morj::plan::Tree*>(tree);
  const ll nn = (ll)t.nodes.size();
  std::vector<int> comp(n_compute);
  for (int i = 0; i < n_compute; ++i) {
    if (compute[i] < 0 || compute[i] >= nn) return morj::set_error(MORJ_ERR_ARG, "morj_plan_pass: bad node id");
    comp[i] = (int)compute[i];
  }
  for (int i = 0; i < n_readout; ++i)
    if (readout_seqs[i] < 0 || readout_seqs[i] >= (int)t.seqs.size())
      return morj::set_error(MORJ_ERR_ARG, "morj_plan_pass: bad sequence index");
  for (ll i = 0; i < n_prealloc; ++i)
    if (prealloc[i] < 0 || prealloc[i] >= t.num_tokens)
      return morj::set_error(MORJ_ERR_ARG, "morj_plan_pass: bad preallocated offset");
  const ll* pins[2] = {pinned_g, pinned_s};
  const ll n_pins[2] = {pinned_g ? n_pinned_g : 0, pinned_s ? n_pinned_s : 0};
  for (int k = 0; k < 2; ++k)
    for (ll i = 0; i < n_pins[k]; ++i)
      if (pins[k][i] < 0 || pins[k][i] >= t.num_tokens)
        return morj::set_error(MORJ_ERR_ARG, "morj_plan_pass: bad pinned offset");
  const ll* init[2] = {initial_g, initial_s};
  std::unordered_set<int> bid;
  for (int i = 0; i < n_bidir; ++i) bid.insert((int)bidir[i]);
  auto* p = new (std::nothrow) morj::plan::Plan;
  if (!p) return morj::set_error(MORJ_ERR_OOM, "morj_plan_pass: out of host memory");
  const int st = morj::plan::plan_pass(t, std::move(comp), readout_seqs, n_readout, window, single_max, step_tokens,
                                       identity, prealloc, n_prealloc, init, pins, n_pins, bid, *p);
  if (st) {
    delete p;
    return st;
  }
  *plan = p;
  return MORJ_OK;
}

extern "C" int morj_plan_blob(const void* plan, const long long** data, long long* len) {
  if (!plan || !data || !len) return morj::set_error(MORJ_ERR_ARG, "morj_plan_blob: bad arguments");
  const auto& p = *static_cast<const morj::plan::Plan*>(plan);
  *data = p.blob.data();
  *len = (ll)p.blob.size();
  return MORJ_OK;
}

extern "C" void morj_plan_free(void* plan) {
  auto* p = static_cast<morj::plan::Plan*>(plan);
  if (!p) return;
  if (morj::plan::t_pool.size() < 4) morj::plan::t_pool.push_back(std::move(p->blob));
  delete p;
}
