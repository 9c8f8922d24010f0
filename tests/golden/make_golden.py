"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in the build container (needs the reference tree and oracle/_ref built by
`make -C oracle ref`):

    python tests/golden/make_golden.py

* c1.json / c1u.json: the reference C++ core (compiled from its own sources) on the
  seeded synthetic tiny target (C1 config; "c1u" = the same with an untied LM head,
  whose greedy stream is not a repeat of the last prompt token). Last-row logits,
  AR greedy tokens, and speculative greedy tokens for chain:4 and tree:3,3,8.
* sampling.json: the reference's Python acceptance functions
  (python/woodcock/sampling.py, imported with an empty stand-in `mlx` module: the
  functions used here are pure numpy) on seeded cases, driven by the Philox uniform
  tape of oracle/wc_oracle.py. Inputs and outputs are stored so the tests can
  replay them against the oracle and the CUDA acceptance kernel.
* c1u_forced.json: the reference C++ core in oracle-drafter mode (`wc_ref_driver forced`) on
  the C1u pair: chains of 4 and 6 with seeded accept lengths and draft trees whose accepted
  paths branch, per round the tree, accepted path, next token, the drafter's own head
  proposals (root and every drafted node) and the cache lengths
  (`python tests/golden/make_golden.py forced`).
* c3_reference.json: the reference C++ core on the full 28-layer C3 target (Qwen3-1.7B
  architecture; the bench's seeded bf16 weights, read by the reference in fp32): its greedy
  continuation of an 8-token prompt and, teacher-forced on it, every row's argmax, top-8
  logits and the logits at 256 seeded ids (`python tests/golden/make_golden.py c3`; needs a
  CUDA device, because the weights are the bench's seeded device stream, and oracle/_ref).
* vocab.json: the reference's top_ids / coverage (python/woodcock/vocab.py:35-52) on
  seeded counts with ties and forced ids (`python tests/golden/make_golden.py vocab`).
"""

from __future__ import annotations

import dataclasses
import json
import os
import subprocess
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF = Path(os.environ.get("WC_REFERENCE_DIR", "/root/reference"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))

import wc_oracle as O  # noqa: E402

from woodcock_b200 import synthetic as syn  # noqa: E402

DRIVER = REPO / "oracle" / "_ref" / "wc_ref_driver"
N_NEW = 128


def _run(*args) -> dict:
    r = subprocess.run([str(DRIVER), *args], capture_output=True, text=True, check=True)
    return json.loads(r.stdout)


def model_fixture(name: str, tie: bool) -> dict:
    ts = dataclasses.replace(syn.TINY_TARGET, tie_embeddings=tie)
    with tempfile.TemporaryDirectory() as tmp:
        td, dd, tw, dw = syn.make_pair(tmp, "c1", seed=0, dtype="F32", target_spec=ts)
        prompt = syn.prompt_ids(64, ts.vocab, seed=0)
        ids = ",".join(map(str, prompt))
        common = ["--target", str(td), "--ids", ids, "--taps", "1,2,3"]
        fwd = _run("forward", *common)
        ar = _run("gen", "--ar", *common, "--max", str(N_NEW))
        out = {
            "config": "c1", "tie_embeddings": tie, "seed": 0, "taps": [1, 2, 3], "prompt": prompt,
            "weights_checksum": float(sum(float(np.abs(v).sum()) for v in tw.values())),
            "last_logits": fwd["last_logits"], "argmax": fwd["argmax"],
            "taps_last_head8": [t[:8] for t in fwd["taps_last"]],
            "ar_tokens": ar["tokens"],
        }
        for pol in ("chain:4", "tree:3,3,8"):
            sd = _run("gen", *common, "--drafter", str(dd), "--max", str(N_NEW), "--policy", pol)
            out[f"spec_{pol}"] = {"tokens": sd["tokens"], "rounds": sd["rounds"], "accepted": sd["accepted"]}
    return out


def chain_template(K: int, accept: int) -> str:
    """K chained drafts; draft accept+1 is corrupted (none when accept == K)."""
    return " ".join(f"{j}:{j}:{1 if j == accept else 0}" for j in range(K))


# Forced draft trees (parent:offset:delta per node, node 0 = the root): the second root child
# accepted with a matching node under the rejected first child; both children of an accepted
# node rejected; nothing accepted; a depth-3 path with a side branch.
FORCED_TREES = ["0:0:1 0:0:0 2:1:0 1:1:0 3:2:1 3:2:0", "0:0:0 1:1:1 1:1:2 3:2:0", "0:0:2 0:0:1 1:1:0",
                "0:0:0 1:1:0 2:2:0 3:3:1 2:2:3"]
FORCED_SETS = {"chain4": [chain_template(4, a) for a in (2, 4, 0, 3, 1)],
               "chain6": [chain_template(6, a) for a in (6, 1, 3, 5, 0)],
               "tree": FORCED_TREES}
FORCED_NEW = 96


def forced_fixture() -> dict:
    ts = dataclasses.replace(syn.TINY_TARGET, tie_embeddings=False)
    out = {"config": "c1u", "taps": [1, 2, 3], "max_new": FORCED_NEW}
    with tempfile.TemporaryDirectory() as tmp:
        td, dd, _, _ = syn.make_pair(tmp, "c1", seed=0, dtype="F32", target_spec=ts)
        prompt = syn.prompt_ids(64, ts.vocab, seed=0)
        out["prompt"] = prompt
        for name, tpl in FORCED_SETS.items():
            f = Path(tmp) / f"{name}.txt"
            f.write_text("\n".join(tpl) + "\n")
            r = _run("forced", "--target", str(td), "--drafter", str(dd), "--ids", ",".join(map(str, prompt)),
                     "--taps", "1,2,3", "--max", str(FORCED_NEW), "--trees", str(f))
            r["templates"] = tpl
            for key in ("round_s", "t_prefill"):  # timings: not part of the fixture
                r.pop(key, None)
            out[name] = r
    return out


C3_PROMPT, C3_NEW, C3_SAMPLE = 8, 16, 256


def c3_fixture() -> dict:
    from woodcock_b200 import synthetic as syn

    ts = syn.Q17_TARGET
    prompt = syn.prompt_ids(C3_PROMPT, ts.vocab, seed=3)
    sample = np.sort(np.random.default_rng(4).choice(ts.vocab, C3_SAMPLE, replace=False)).tolist()
    with tempfile.TemporaryDirectory() as tmp:
        td = syn.write_device_model(Path(tmp) / "target", ts.hf_config(), syn.target_tensor_specs(ts), 0)
        common = ["--target", str(td), "--taps", "2,14,26"]
        ar = _run("gen", "--ar", *common, "--ids", ",".join(map(str, prompt)), "--max", str(C3_NEW), "--no-eos")
        seq = prompt + ar["tokens"][: C3_NEW - 1]
        fw = _run("forward", *common, "--ids", ",".join(map(str, seq)), "--rows-from", str(C3_PROMPT - 1),
                  "--top", "8", "--sample-ids", ",".join(map(str, sample)))
    return {"config": "c3 target (Qwen3-1.7B architecture, 28 layers), device weight stream seed 0",
            "prompt": prompt, "ar_tokens": ar["tokens"], "sample_ids": sample, "rows": fw["rows"]}


def _reference_sampling():
    stub = types.ModuleType("mlx")
    stub.core = types.ModuleType("mlx.core")
    sys.modules.setdefault("mlx", stub)
    sys.modules.setdefault("mlx.core", stub.core)
    sys.path.insert(0, str(REF / "python"))
    from woodcock import sampling as ref_sampling  # noqa: E402

    return ref_sampling


def sampling_fixture() -> dict:
    S = _reference_sampling()
    rs = np.random.default_rng(123)
    cases = {"chain": [], "tree": [], "greedy_tree": [], "mask": [], "gumbel": []}
    V = 11
    for i in range(40):
        K = int(rs.integers(1, 5))
        p = rs.dirichlet(np.full(V, 0.6), size=K + 1)
        q = rs.dirichlet(np.full(V, 0.6), size=K)
        if i % 4 == 1:  # truncated draft vocabulary: q = 0 on the top ids
            q[:, V - 3:] = 0.0
            q /= q.sum(-1, keepdims=True)
        if i % 5 == 2:  # a near-identical pair exercises the residual fallback
            q[0] = p[0]
        toks = [int(np.argmax(rs.multinomial(1, qq))) for qq in q]
        seed = 1000 + i
        tape = O.Tape(seed)
        n, nxt = S.verify_chain_stochastic(p, q, toks, tape)
        cases["chain"].append({"p": p.tolist(), "q": q.tolist(), "tokens": toks, "seed": seed,
                               "accepted": int(n), "next": int(nxt), "uniforms_used": tape.pos})
    for i in range(24):
        depth, width = int(rs.integers(1, 3)), int(rs.integers(1, 4))
        tokens, parents, depths = [int(rs.integers(V))], [-1], [0]
        frontier, qd = [0], {}
        seed = 5000 + i
        tape = O.Tape(seed)
        for dd in range(1, depth + 1):
            nxt_f = []
            for v in frontier:
                qv = rs.dirichlet(np.full(V, 0.7))
                qd[v] = qv
                for x in S.sample_without_replacement(qv, width, tape):
                    tokens.append(int(x)); parents.append(v); depths.append(dd)
                    nxt_f.append(len(tokens) - 1)
            frontier = nxt_f
        p = rs.dirichlet(np.full(V, 0.7), size=len(tokens))
        tree = S.DraftTree(tokens, parents, depths)
        path, nxt = S.verify_tree_stochastic({v: p[v] for v in range(len(tokens))}, qd, tree, tape)
        cases["tree"].append({"tokens": tokens, "parents": parents, "depth": depths, "p": p.tolist(),
                              "q": {str(k): v.tolist() for k, v in qd.items()}, "seed": seed,
                              "path": [int(x) for x in path], "next": int(nxt), "uniforms_used": tape.pos})
    for i in range(24):
        n_nodes = int(rs.integers(2, 12))
        parents = [-1] + [int(rs.integers(0, v)) for v in range(1, n_nodes)]
        depth = [0] * n_nodes
        for v in range(1, n_nodes):
            depth[v] = depth[parents[v]] + 1
        tokens = [int(rs.integers(0, 6)) for _ in range(n_nodes)]
        am = [int(rs.integers(0, 6)) for _ in range(n_nodes)]
        tree = S.DraftTree(tokens, parents, depth)
        path, nxt = S.verify_tree_greedy(am, tree)
        cases["greedy_tree"].append({"tokens": tokens, "parents": parents, "depth": depth, "argmax": am,
                                     "path": [int(x) for x in path], "next": int(nxt)})
        prefix = int(rs.integers(0, 5))
        cases["mask"].append({"parents": parents, "tokens": tokens, "depth": depth, "prefix": prefix,
                              "mask": S.tree_attention_mask(tree, prefix).astype(int).tolist()})
    for i in range(8):
        q = rs.dirichlet(np.full(V, 0.5))
        q[rs.integers(V)] = 0.0
        seed = 9000 + i
        tape = O.Tape(seed)
        k = int(rs.integers(1, 4))
        cases["gumbel"].append({"q": q.tolist(), "k": k, "seed": seed,
                                "out": S.sample_without_replacement(q, k, tape), "uniforms_used": tape.pos})
    return cases


def vocab_fixture() -> dict:
    """python/woodcock/vocab.py:35-47 top_ids on seeded counts with many ties and forced ids."""
    _reference_sampling()  # puts the reference package on the path (with the stand-in mlx)
    from woodcock import vocab as ref_vocab  # noqa: E402

    rs = np.random.default_rng(7)
    cases = []
    for i in range(30):
        V = int(rs.integers(5, 400))
        counts = rs.integers(0, 6 if i % 2 else 1000, V)
        k = int(rs.integers(1, V + 1))
        always = sorted({int(x) for x in rs.integers(0, V, int(rs.integers(0, min(k, 4) + 1)))})
        ids = ref_vocab.top_ids(counts, k, set(always))
        cases.append({"counts": counts.tolist(), "k": k, "always": always, "ids": ids.tolist(),
                      "coverage": ref_vocab.coverage(counts, ids)})
    return {"top_ids": cases}


def main():
    only = sys.argv[1:]
    if not only or "models" in only:
        for name, tie in (("c1", True), ("c1u", False)):
            (HERE / f"{name}.json").write_text(json.dumps(model_fixture(name, tie)))
            print("wrote", name)
    if not only or "sampling" in only:
        (HERE / "sampling.json").write_text(json.dumps(sampling_fixture()))
        print("wrote sampling")
    if not only or "forced" in only:
        (HERE / "c1u_forced.json").write_text(json.dumps(forced_fixture()))
        print("wrote c1u_forced")
    if "c3" in only:  # needs a CUDA device: not part of the default run
        (HERE / "c3_reference.json").write_text(json.dumps(c3_fixture()))
        print("wrote c3_reference")
    if not only or "vocab" in only:
        (HERE / "vocab.json").write_text(json.dumps(vocab_fixture()))
        print("wrote vocab")


if __name__ == "__main__":
    main()
