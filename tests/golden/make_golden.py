"""Generate the golden fixtures in this directory by running the reference
engine itself (vedantjain09/paged-speculative-engine, pure Python / PyTorch).

The reference is only importable where its source tree is present; the
fixtures it produces are committed so the tests can check the oracle and the
CUDA path without it.  Run from the repository root:

    python tests/golden/make_golden.py <reference checkout>

Fixtures:

* ``init_checksums.json``  sha256 of the state_dict of reference-constructed
  TinyGPT models (seeded), to pin that the restated constructor draws the same
  weights;
* ``tiny_greedy.json``     the "tiny" workload (TinyGPT pair, 8 prompts, 64 new,
  k=4, block 16, batch 4, T=0) through the reference scheduler: every request's
  output, ``generate_cached`` of every prompt, and after every scheduler step
  the per-request accepted tokens plus both caches' block tables, lengths and
  free lists;
* ``tiny_logits.json``     the target's last-position logits of each prompt
  (full forward, fp32);
* ``cache_ops.json``       a seeded random create/append/truncate/free sequence
  on the reference PagedKVCache with the state after every operation;
* ``first_token_dists.json`` the exact first-token target distributions of the
  two chi-squared models of the reference's distribution tests.
"""
from __future__ import annotations

import hashlib
import json
import os
import random
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _state_sha(model) -> str:
    h = hashlib.sha256()
    for name, t in model.state_dict().items():
        h.update(name.encode())
        h.update(t.detach().contiguous().float().numpy().tobytes())
    return h.hexdigest()


def _cache_state(cache) -> dict:
    return {
        "tables": {rid: list(t) for rid, t in cache._block_tables.items()},
        "lengths": dict(cache._lengths),
        "free": list(cache.allocator._free),
    }


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(REPO, "paged-speculative-engine_b200"))
    from engine.generate import generate_cached  # noqa: E402  (reference)
    from engine.model import ModelConfig, TinyGPT  # noqa: E402
    from engine.paged_cache import PagedKVCache  # noqa: E402
    from engine.scheduler import Request, run_continuous_speculative_batches  # noqa: E402
    import engine.speculative as ref_spec  # noqa: E402
    from pse import workload as wl  # noqa: E402

    torch.set_num_threads(1)

    # 1. constructor pins
    cases = [
        dict(seed=0, cfg=dict(vocab_size=64, d_model=16, n_layers=2, n_heads=2, d_ff=32, max_seq_len=128)),
        dict(seed=3, cfg=dict(vocab_size=48, d_model=12, n_layers=2, n_heads=2, d_ff=32, max_seq_len=128)),
        dict(seed=7, cfg=dict(vocab_size=32, d_model=12, n_layers=2, n_heads=2, d_ff=24, max_seq_len=256)),
    ]
    out = []
    for c in cases:
        torch.manual_seed(c["seed"])
        a = TinyGPT(ModelConfig(**c["cfg"]))
        b = TinyGPT(ModelConfig(**c["cfg"]))
        out.append(dict(c, sha_first=_state_sha(a), sha_second=_state_sha(b)))
    tiny = wl.WORKLOADS["tiny"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.draft))
    t = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.target))
    out.append(dict(seed=0, workload="tiny", sha_draft=_state_sha(d), sha_target=_state_sha(t)))
    with open(os.path.join(HERE, "init_checksums.json"), "w") as f:
        json.dump(out, f, indent=1)

    # 2. tiny workload through the reference scheduler, with per-step state
    d.eval()
    t.eval()
    prompts = wl.prompts(tiny, seed=0)
    rids = wl.request_ids(len(prompts))
    bs = tiny.block_size
    num_blocks = 96
    dc = PagedKVCache(tiny.pair.draft["n_layers"], tiny.pair.draft["n_heads"],
                      tiny.pair.draft["d_model"] // tiny.pair.draft["n_heads"], bs, num_blocks)
    tc = PagedKVCache(tiny.pair.target["n_layers"], tiny.pair.target["n_heads"],
                      tiny.pair.target["d_model"] // tiny.pair.target["n_heads"], bs, num_blocks)
    steps = []
    real_step = ref_spec.batched_speculative_step

    def traced_step(*args, **kwargs):
        res = real_step(*args, **kwargs)
        ids = args[2]
        steps.append(dict(ids=list(ids),
                          accepted={r: res.accepted_tokens[r] for r in ids},
                          n_acc={r: res.num_draft_accepted[r] for r in ids},
                          draft=_cache_state(dc), target=_cache_state(tc)))
        return res

    import engine.scheduler as ref_sched
    ref_sched.batched_speculative_step = traced_step
    try:
        reqs = [Request(r, p, tiny.max_new_tokens) for r, p in zip(rids, prompts)]
        results = run_continuous_speculative_batches(d, t, reqs, dc, tc, tiny.max_batch_size,
                                                     k=tiny.k, temperature=0.0)
    finally:
        ref_sched.batched_speculative_step = real_step
    baselines = {r: generate_cached(t, torch.tensor([p]), tiny.max_new_tokens) for r, p in zip(rids, prompts)}
    golden = dict(
        workload="tiny", num_blocks=num_blocks, prompts=prompts, request_ids=rids,
        outputs={res.request_id: res.output_ids for res in results},
        generate_cached=baselines, steps=steps,
        final_free={"draft": list(dc.allocator._free), "target": list(tc.allocator._free)},
    )
    with open(os.path.join(HERE, "tiny_greedy.json"), "w") as f:
        json.dump(golden, f)

    # 3. last-position logits of each prompt
    with torch.no_grad():
        logits = [t(torch.tensor([p]))[0][0, -1].tolist() for p in prompts]
    with open(os.path.join(HERE, "tiny_logits.json"), "w") as f:
        json.dump(dict(prompts=prompts, logits=logits), f)

    # 4. random cache operation sequences (the second pool is small enough to
    #    run dry: the state after each MemoryError is recorded as it stands)
    seqs = []
    for seed, nb in ((1234, 24), (99, 8)):
        rng = random.Random(seed)
        cache = PagedKVCache(1, 1, 2, 4, nb)
        alive: list[str] = []
        ops, states = [], []
        counter = 0
        for _ in range(300):
            kind = rng.choice(["append", "append", "truncate", "free", "create"])
            if kind == "create" or not alive:
                rid = f"q{counter}"
                counter += 1
                cache.create_request(rid)
                alive.append(rid)
                ops.append(["create", rid, 0])
            elif kind == "append":
                rid = rng.choice(alive)
                n = rng.randint(1, 7)
                try:
                    cache.append(rid, [torch.full((1, n, 2), 1.0)], [torch.full((1, n, 2), 1.0)])
                    ops.append(["append", rid, n])
                except MemoryError:
                    ops.append(["append_oom", rid, n])
            elif kind == "truncate":
                rid = rng.choice(alive)
                n = rng.randint(0, cache.length(rid))
                cache.truncate(rid, n)
                ops.append(["truncate", rid, n])
            else:
                rid = rng.choice(alive)
                cache.free_request(rid)
                alive.remove(rid)
                ops.append(["free", rid, 0])
            states.append(_cache_state(cache))
        seqs.append(dict(num_blocks=nb, block_size=4, ops=ops, states=states))
    with open(os.path.join(HERE, "cache_ops.json"), "w") as f:
        json.dump(seqs, f)

    # 5. chi-squared reference distributions (tests/test_distribution_preserving.py:30-43)
    dists = []
    for seed, prompt in ((10, [1, 2, 3]), (11, [2, 4, 1])):
        torch.manual_seed(seed)
        cfg = ModelConfig(vocab_size=12, d_model=8, n_layers=1, n_heads=2, d_ff=16, max_seq_len=32)
        TinyGPT(cfg)
        target = TinyGPT(cfg)
        with torch.no_grad():
            lg = target(torch.tensor([prompt]))[0][0, -1]
        dists.append(dict(seed=seed, prompt=prompt, probs=torch.softmax(lg, -1).tolist()))
    with open(os.path.join(HERE, "first_token_dists.json"), "w") as f:
        json.dump(dists, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout (its engine/ package)>")
    main(sys.argv[1])
