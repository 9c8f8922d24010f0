// Test-infrastructure driver around the reference C++ core (built from the
// reference's own sources by oracle/Makefile into oracle/_ref/). It is the
// checker for the CUDA path and the timed CPU baseline; nothing in the
// product links or calls it.
//
// It drives the reference's public C++ API exactly as its own CLI does
// (tools/woodcock_generate.cpp:23-71), plus the two things that CLI cannot
// do: explicit target taps (Qwen3(dir, taps), include/woodcock/model.h:36)
// and dumping the target forward's last-row logits / taps.
//
//   wc_ref_driver gen     --target D [--drafter D] --ids 1,2 [--max N] [--policy chain:K|tree:D,W,N]
//                         [--taps a,b,c] [--temp T] [--seed S] [--ar] [--no-eos]
//   wc_ref_driver forward --target D --ids 1,2 [--taps a,b,c] [--rows-from R --top K --sample-ids a,b]
//   wc_ref_driver forced  --target D --drafter D --ids 1,2 --max N --trees FILE [--taps a,b,c]
// Output: one JSON object on stdout.
//
// `forward --rows-from R` (for large vocabularies) prints, instead of the last row's full
// logits, for every row r >= R: the argmax, the top K ids and logits (largest first) and
// the logits at the given sample ids.
//
// `forced` is the oracle-drafter mode (the OracleDecoder pattern of the reference's
// tests/test_spec_model.py:59-92) run on the reference's own C++ functions. The reference's
// greedy continuation A (generate_autoregressive) is computed first; each round then verifies a
// draft tree whose tokens come from a template in FILE instead of from the drafter. A template
// line lists nodes 1..N-1 as "parent:offset:delta": the node's token is A[e + offset] + delta
// (mod vocab; delta 0 = the continuation itself), where e = tokens emitted so far; round r uses template
// r mod (lines). The round follows SpeculativeDecoder's draft / verify / update
// (src/core/spec.cpp:86-233) step for step with those tokens: the drafter still runs over
// every internal node of the tree (positions n-1+depth, mask = committed entries + drafted
// ancestors + itself, spec.cpp:158-171) and its own proposal (head argmax) and largest logit
// are recorded for the root and every drafted node; the target verifies with positions
// n+depth and tree_mask (chains: the plain causal forward), verify_tree_greedy picks the
// path, KVCache::compact keeps it, and the drafter is updated on the accepted rows.
#include <chrono>
#include <cstdio>
#include <fstream>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "woodcock/spec.h"

using namespace woodcock;

static std::vector<int> parse_ints(const std::string& s) {
  std::vector<int> v;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ','))
    if (!tok.empty()) v.push_back(std::stoi(tok));
  return v;
}

static void print_ints(const char* key, const std::vector<int>& v) {
  std::printf("\"%s\": [", key);
  for (size_t i = 0; i < v.size(); ++i) std::printf("%s%d", i ? ", " : "", v[i]);
  std::printf("]");
}

static void print_floats(const char* key, const float* v, size_t n) {
  std::printf("\"%s\": [", key);
  for (size_t i = 0; i < n; ++i) std::printf("%s%.9g", i ? ", " : "", double(v[i]));
  std::printf("]");
}

namespace {

struct TemplateNode {
  int parent, offset, delta;
};

std::vector<std::vector<TemplateNode>> read_templates(const std::string& path) {
  std::vector<std::vector<TemplateNode>> out;
  std::ifstream f(path);
  if (!f) {
    std::fprintf(stderr, "cannot read %s\n", path.c_str());
    std::exit(2);
  }
  std::string line;
  while (std::getline(f, line)) {
    std::stringstream ss(line);
    std::string item;
    std::vector<TemplateNode> t;
    while (ss >> item) {
      TemplateNode nd{};
      if (std::sscanf(item.c_str(), "%d:%d:%d", &nd.parent, &nd.offset, &nd.delta) != 3) {
        std::fprintf(stderr, "bad template node %s\n", item.c_str());
        std::exit(2);
      }
      if (nd.parent < 0 || nd.parent > int(t.size())) {
        std::fprintf(stderr, "template node parent %d must precede the node\n", nd.parent);
        std::exit(2);
      }
      t.push_back(nd);
    }
    if (!t.empty()) out.push_back(t);
  }
  if (out.empty()) {
    std::fprintf(stderr, "no templates in %s\n", path.c_str());
    std::exit(2);
  }
  return out;
}

// The drafter's own choice on one output row: head argmax and its logit.
void propose(const Drafter& d, const float* out_row, int* tok, float* zmax) {
  std::vector<float> z;
  d.logits(out_row, z);
  *tok = argmax(z.data(), int(z.size()));
  *zmax = z[size_t(*tok)];
}

int run_forced(const Qwen3& t, const Drafter& d, const std::vector<int>& prompt, int max_new,
               const std::string& trees_path) {
  const auto tpl = read_templates(trees_path);
  const int V = t.config().vocab, Dt = t.config().hidden, dd = d.config().hidden, window = d.config().window;
  int max_off = 0;
  for (const auto& tp : tpl)
    for (const auto& nd : tp) max_off = std::max(max_off, nd.offset);
  SamplingParams greedy;
  GenStats ar_st;
  const std::vector<int> A = generate_autoregressive(t, prompt, max_new + max_off + 2, greedy, &ar_st, {});

  // prefill (spec.cpp:61-84)
  const auto t_pre0 = std::chrono::steady_clock::now();
  KVCache tc = t.make_cache(), dc = d.make_cache();
  const int np = int(prompt.size());
  ForwardArgs fa;
  fa.logits_from = np - 1;
  ForwardOut o = t.forward(prompt, tc, fa);
  const int first = argmax(o.logits.data(), V);
  std::vector<int> shifted(prompt.begin() + 1, prompt.end());
  shifted.push_back(first);
  DraftOut od = d.forward(shifted, d.fuse(o.taps, np), dc);
  std::vector<float> root_out(od.out.end() - dd, od.out.end());
  std::vector<float> root_fb(d.feedback_row(od, np - 1), d.feedback_row(od, np - 1) + dd);

  const double t_prefill = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_pre0).count();
  std::vector<int> out{first};
  std::vector<float> round_s;
  long accepted = 0;
  std::printf("{\"first\": %d, ", first);
  print_ints("ar", A);
  std::printf(", \"rounds\": [");
  for (int r = 0; int(out.size()) < max_new; ++r) {
    const auto t_r0 = std::chrono::steady_clock::now();
    const int n = tc.size(), e = int(out.size());
    const auto& tp = tpl[size_t(r) % tpl.size()];
    DraftTree tree;
    tree.tokens.push_back(out.back());
    tree.parents.push_back(-1);
    tree.depth.push_back(0);
    for (const auto& nd : tp) {
      const int tok = (A[size_t(e + nd.offset)] + nd.delta) % V;
      tree.tokens.push_back(tok);
      tree.parents.push_back(nd.parent);
      tree.depth.push_back(tree.depth[size_t(nd.parent)] + 1);
    }
    tree.build_children();
    const int N = tree.size();
    int max_depth = 0;
    for (int v = 0; v < N; ++v) max_depth = std::max(max_depth, tree.depth[size_t(v)]);

    // drafting over the given tree: proposals of the root and of every drafted node
    std::vector<std::vector<float>> outs(static_cast<size_t>(N)), fbs(static_cast<size_t>(N));
    std::vector<int> cache_idx(static_cast<size_t>(N), -1), prop_tok(static_cast<size_t>(N), -1);
    std::vector<float> prop_z(static_cast<size_t>(N), 0.f);
    outs[0] = root_out;
    fbs[0] = root_fb;
    cache_idx[0] = n - 1;
    propose(d, outs[0].data(), &prop_tok[0], &prop_z[0]);
    const int base = dc.size();
    int drafted = 0;
    for (int depth = 1; depth < max_depth; ++depth) {
      std::vector<int> level;
      for (int v = 1; v < N; ++v)
        if (tree.depth[size_t(v)] == depth && !tree.children[size_t(v)].empty()) level.push_back(v);
      if (level.empty()) break;
      const int m = int(level.size()), T = base + drafted + m;
      std::vector<int> toks, pos;
      std::vector<float> fb(size_t(m) * dd);
      std::vector<uint8_t> mask(size_t(m) * T, 0);
      for (int i = 0; i < m; ++i) {
        const int v = level[size_t(i)];
        toks.push_back(tree.tokens[size_t(v)]);
        pos.push_back(n - 1 + depth);
        std::copy(fbs[size_t(tree.parents[size_t(v)])].begin(), fbs[size_t(tree.parents[size_t(v)])].end(),
                  fb.begin() + int64_t(i) * dd);
        const int p = base - 1 + depth;
        const int lo = window > 0 ? std::max(0, p - window + 1) : 0;
        for (int c = lo; c < base; ++c) mask[size_t(i) * T + c] = 1;
        for (int u = tree.parents[size_t(v)]; u > 0; u = tree.parents[size_t(u)]) mask[size_t(i) * T + cache_idx[size_t(u)]] = 1;
        mask[size_t(i) * T + base + drafted + i] = 1;
      }
      DraftOut dr = d.forward(toks, fb, dc, &pos, &mask);
      for (int i = 0; i < m; ++i) {
        const int v = level[size_t(i)];
        outs[size_t(v)].assign(dr.out.begin() + int64_t(i) * dd, dr.out.begin() + int64_t(i + 1) * dd);
        fbs[size_t(v)].assign(d.feedback_row(dr, i), d.feedback_row(dr, i) + dd);
        cache_idx[size_t(v)] = base + drafted + i;
        propose(d, outs[size_t(v)].data(), &prop_tok[size_t(v)], &prop_z[size_t(v)]);
      }
      drafted += m;
    }
    dc.trim_to(base);

    // verification (spec.cpp:189-224)
    ForwardOut vo;
    if (tree.is_chain()) {
      vo = t.forward(tree.tokens, tc);
    } else {
      std::vector<int> pos;
      for (int dpt : tree.depth) pos.push_back(n + dpt);
      const auto mask = tree_mask(tree, n);
      ForwardArgs a;
      a.positions = &pos;
      a.mask = &mask;
      vo = t.forward(tree.tokens, tc, a);
    }
    std::vector<int> am(static_cast<size_t>(N));
    for (int v = 0; v < N; ++v) am[size_t(v)] = argmax(vo.logits.data() + int64_t(v) * V, V);
    const Verdict verdict = verify_tree_greedy(am, tree);
    std::vector<int> keep{0};
    keep.insert(keep.end(), verdict.path.begin(), verdict.path.end());
    tc.compact(n, keep);
    std::vector<std::vector<float>> taps(vo.taps.size());
    for (size_t f = 0; f < vo.taps.size(); ++f)
      for (int v : keep)
        taps[f].insert(taps[f].end(), vo.taps[f].begin() + int64_t(v) * Dt, vo.taps[f].begin() + int64_t(v + 1) * Dt);

    // drafter update on the accepted rows (spec.cpp:226-233)
    std::vector<int> acc;
    for (int v : verdict.path) acc.push_back(tree.tokens[size_t(v)]);
    acc.push_back(verdict.next);
    DraftOut uo = d.forward(acc, d.fuse(taps, int(acc.size())), dc);
    root_out.assign(uo.out.end() - dd, uo.out.end());
    root_fb.assign(d.feedback_row(uo, int(acc.size()) - 1), d.feedback_row(uo, int(acc.size()) - 1) + dd);
    accepted += long(verdict.path.size());
    round_s.push_back(float(std::chrono::duration<double>(std::chrono::steady_clock::now() - t_r0).count()));

    std::printf("%s{", r ? ", " : "");
    print_ints("tokens", tree.tokens);
    std::printf(", ");
    print_ints("parents", tree.parents);
    std::printf(", ");
    print_ints("path", verdict.path);
    std::printf(", \"next\": %d, ", verdict.next);
    print_ints("proposals", prop_tok);
    std::printf(", ");
    print_floats("proposal_logits", prop_z.data(), prop_z.size());
    std::printf(", \"n\": %d, \"drafter_len\": %d}", tc.size(), dc.size());
    for (int tok : acc) {
      if (int(out.size()) >= max_new) break;
      out.push_back(tok);
    }
  }
  std::printf("], ");
  print_ints("tokens", out);
  std::printf(", \"accepted\": %ld, \"t_prefill\": %.6f, ", accepted, t_prefill);
  print_floats("round_s", round_s.data(), round_s.size());
  std::printf("}\n");
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: wc_ref_driver gen|forward --target DIR ...\n");
    return 2;
  }
  const std::string cmd = argv[1];
  std::string target, drafter, ids, policy = "chain:4", taps_s, trees, sample_s;
  int rows_from = -1, top = 8;
  int max_new = 128;
  float temp = 0.f;
  unsigned long long seed = 0;
  bool ar = false, no_eos = false;
  for (int i = 2; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) { std::fprintf(stderr, "missing value for %s\n", a.c_str()); std::exit(2); }
      return std::string(argv[++i]);
    };
    if (a == "--target") target = next();
    else if (a == "--drafter") drafter = next();
    else if (a == "--ids") ids = next();
    else if (a == "--max") max_new = std::stoi(next());
    else if (a == "--policy") policy = next();
    else if (a == "--taps") taps_s = next();
    else if (a == "--temp") temp = std::stof(next());
    else if (a == "--seed") seed = std::stoull(next());
    else if (a == "--ar") ar = true;
    else if (a == "--no-eos") no_eos = true;
    else if (a == "--trees") trees = next();
    else if (a == "--rows-from") rows_from = std::stoi(next());
    else if (a == "--top") top = std::stoi(next());
    else if (a == "--sample-ids") sample_s = next();
    else { std::fprintf(stderr, "unknown argument %s\n", a.c_str()); return 2; }
  }
  if (target.empty() || ids.empty()) {
    std::fprintf(stderr, "--target and --ids are required\n");
    return 2;
  }
  std::array<int, 3> taps{-1, -1, -1};
  if (!taps_s.empty()) {
    auto t = parse_ints(taps_s);
    if (t.size() != 3) { std::fprintf(stderr, "--taps needs three layer indices\n"); return 2; }
    taps = {t[0], t[1], t[2]};
  }
  const auto t_load0 = std::chrono::steady_clock::now();
  Qwen3 t(target, taps);
  const std::vector<int> prompt = parse_ints(ids);

  if (cmd == "forward" && rows_from >= 0) {
    KVCache c = t.make_cache();
    ForwardArgs a;
    const int L = int(prompt.size()), V = t.config().vocab;
    if (rows_from >= L) { std::fprintf(stderr, "--rows-from must be below the number of ids\n"); return 2; }
    a.logits_from = rows_from;
    const ForwardOut o = t.forward(prompt, c, a);
    const std::vector<int> sample = parse_ints(sample_s);
    std::printf("{\"rows\": [");
    for (int r = rows_from; r < L; ++r) {
      const float* z = o.logits.data() + int64_t(r - rows_from) * V;
      std::vector<int> order(static_cast<size_t>(V));
      for (int i = 0; i < V; ++i) order[size_t(i)] = i;
      const int k = std::min(top, V);
      std::partial_sort(order.begin(), order.begin() + k, order.end(),
                        [&](int x, int y) { return z[x] != z[y] ? z[x] > z[y] : x < y; });
      order.resize(size_t(k));
      std::vector<float> tv, sv;
      for (int i : order) tv.push_back(z[i]);
      for (int i : sample) sv.push_back(i >= 0 && i < V ? z[i] : 0.f);
      std::printf("%s{\"row\": %d, \"argmax\": %d, ", r > rows_from ? ", " : "", r, argmax(z, V));
      print_ints("top_ids", order);
      std::printf(", ");
      print_floats("top_logits", tv.data(), tv.size());
      std::printf(", ");
      print_floats("sample_logits", sv.data(), sv.size());
      std::printf("}");
    }
    std::printf("]}\n");
    return 0;
  }
  if (cmd == "forward") {
    KVCache c = t.make_cache();
    ForwardArgs a;
    a.logits_from = int(prompt.size()) - 1;
    ForwardOut o = t.forward(prompt, c, a);
    const int V = t.config().vocab, d = t.config().hidden, L = int(prompt.size());
    std::printf("{");
    print_floats("last_logits", o.logits.data(), size_t(V));
    std::printf(", \"argmax\": %d, \"taps_last\": [", argmax(o.logits.data(), V));
    for (size_t f = 0; f < o.taps.size(); ++f) {
      std::printf("%s[", f ? ", " : "");
      const float* row = o.taps[f].data() + int64_t(L - 1) * d;
      for (int i = 0; i < d; ++i) std::printf("%s%.9g", i ? ", " : "", double(row[i]));
      std::printf("]");
    }
    std::printf("]}\n");
    return 0;
  }
  if (cmd == "forced") {
    if (drafter.empty() || trees.empty()) { std::fprintf(stderr, "forced needs --drafter and --trees\n"); return 2; }
    Drafter dr(drafter);
    return run_forced(t, dr, prompt, max_new, trees);
  }
  if (cmd != "gen") {
    std::fprintf(stderr, "unknown command %s\n", cmd.c_str());
    return 2;
  }
  const std::vector<int> eos = no_eos ? std::vector<int>{} : std::vector<int>{151645, 151643};
  SamplingParams sp;
  sp.temperature = temp;
  sp.seed = seed;
  GenStats st;
  std::vector<int> out;
  std::unique_ptr<Drafter> d;
  std::unique_ptr<Policy> pol;
  if (!ar) {
    if (drafter.empty()) { std::fprintf(stderr, "--drafter is required without --ar\n"); return 2; }
    d = std::make_unique<Drafter>(drafter);
    auto colon = policy.find(':');
    std::string kind = policy.substr(0, colon), arg = colon == std::string::npos ? "" : policy.substr(colon + 1);
    if (kind == "chain") pol = std::make_unique<StaticPolicy>(std::stoi(arg));
    else if (kind == "tree") {
      auto v = parse_ints(arg);
      if (v.size() != 3) { std::fprintf(stderr, "tree policy needs D,W,N\n"); return 2; }
      pol = std::make_unique<StaticPolicy>(v[0], v[1], v[2]);
    } else {
      std::fprintf(stderr, "unknown policy %s\n", policy.c_str());
      return 2;
    }
  }
  const double load_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_load0).count();
  if (ar) {
    out = generate_autoregressive(t, prompt, max_new, sp, &st, eos);
  } else {
    SpeculativeDecoder dec(t, *d, *pol);
    out = dec.generate(prompt, max_new, sp, &st, eos);
  }
  std::printf("{");
  print_ints("tokens", out);
  std::printf(", \"new_tokens\": %d, \"rounds\": %d, \"accepted\": %ld, \"verified\": %ld, \"tokens_per_round\": %.6f,"
              " \"decode_tps\": %.6f, \"t_prefill\": %.6f, \"t_draft\": %.6f, \"t_verify\": %.6f, \"t_update\": %.6f,"
              " \"t_total\": %.6f, \"t_load\": %.6f}\n",
              st.new_tokens, st.rounds, st.accepted, st.verified, st.tokens_per_round(), st.decode_tps(), st.t_prefill,
              st.t_draft, st.t_verify, st.t_update, st.t_total, load_s);
  return 0;
}
