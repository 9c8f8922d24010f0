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
//   wc_ref_driver forward --target D --ids 1,2 [--taps a,b,c]
// Output: one JSON object on stdout.
#include <chrono>
#include <cstdio>
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

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: wc_ref_driver gen|forward --target DIR ...\n");
    return 2;
  }
  const std::string cmd = argv[1];
  std::string target, drafter, ids, policy = "chain:4", taps_s;
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
