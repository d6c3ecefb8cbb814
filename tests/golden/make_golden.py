"""Generates the golden fixtures in tests/golden/ from the REFERENCE itself.

Run where the reference tree is available, with $BPKV_REFERENCE set to it (the
directory that holds core/); the fixtures are committed, the reference is never
read at test time.  `python tests/golden/make_golden.py [page16 compress perhead
score budget writeback]` regenerates the named groups (all by default).

  * page16_*.npz  — outputs of the reference Triton kernel ``_page16_decode_kernel``
    (core/page16_native.py:17-80) executed by Triton's CPU interpreter
    (TRITON_INTERPRET=1), on the seeded inputs of tests/golden/inputs.py.
  * compress_*.npz — ``BlockAlignedSnapKV.compress`` (core/compress.py:64-175)
    run unmodified on CPU: retained_block_idx, debug fields, a checksum of K_final.
  * compress_perhead_*.npz — the same, run once per KV head on that head alone (its
    K/V and the query heads of its group): the per-KV-head selection mode's golden.
  * score_*.npz — block scores of ``KVScheduler._score_layer_blocks_for_selection``
    (core/scheduler.py:565-592), executed with its hard-coded CUDA device
    redirected to the CPU.
  * budget.json — ``KVScheduler._selection_budget_blocks`` (core/scheduler.py:547-564)
    over a grid of lengths / budgets.
  * writeback_*.npz — pool pages written by ``_write_selected_layer_to_pool``
    (core/scheduler.py:735-799) into a CPU pool, aligned and unaligned cases.
"""
from __future__ import annotations

import json
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from tests.golden.inputs import PAGE16_CASES, checksum, compress_case, page16_case  # noqa: E402

if "BPKV_REFERENCE" not in os.environ:
    raise SystemExit("set BPKV_REFERENCE to the reference checkout (the directory that holds core/)")
REF = Path(os.environ["BPKV_REFERENCE"]) / "core"
sys.path.insert(0, str(REF))


def gen_page16():
    import page16_native as ref  # reference module, unmodified
    assert ref.HAS_TRITON
    for name, cfg in PAGE16_CASES.items():
        q, k, v, bt, lens = page16_case(**cfg)
        d = cfg["d"]
        n_rep = cfg["hq"] // cfg["hkv"]
        scale = 1.0 / np.sqrt(d)
        out = ref.page16_decode_attention(
            torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(bt),
            torch.from_numpy(lens), softmax_scale=float(scale), n_rep=n_rep)
        np.savez_compressed(HERE / f"page16_{name}.npz", out=out.float().numpy(),
                            inputs_sha=checksum(q, k, v, bt, lens), scale=scale, n_rep=n_rep)
        print("page16", name, out.shape)


COMPRESS_CASES = {
    # benchmarks/test_block_alignment_regression.py:15-47 shape (fixed budget, partial mid block)
    "regression_l2795": dict(case=dict(seed=7, h_kv=8, L=2795, d=32, n_rep=4, window=16),
                             params=dict(block_size=16, sink_len=16, obs_len=16, retain_budget_tokens=2048)),
    # benchmarks/tests.py:36-54 shape (ratio 0.2, sink=obs=64), smaller L for CPU time
    "ratio_l4100": dict(case=dict(seed=11, h_kv=8, L=4100, d=64, n_rep=4, window=64),
                        params=dict(block_size=16, sink_len=64, obs_len=64, retain_ratio=0.20)),
    # hot blocks, ratio 0.25
    "hot_l8192": dict(case=dict(seed=5, h_kv=8, L=8192, d=128, n_rep=4, window=64, hot_blocks=16, sink=64),
                      params=dict(block_size=16, sink_len=64, obs_len=64, retain_ratio=0.25)),
    # input shorter than the budget: compression skipped
    "skip_le_budget": dict(case=dict(seed=3, h_kv=2, L=600, d=32, n_rep=2, window=16),
                           params=dict(block_size=16, sink_len=16, obs_len=16, retain_budget_tokens=1024)),
}


def gen_compress():
    from compress import BlockAlignedSnapKV
    for name, spec in COMPRESS_CASES.items():
        K, V, Q, hot = compress_case(**spec["case"])
        n_rep = spec["case"]["n_rep"]
        c = BlockAlignedSnapKV(**spec["params"])
        Kf, Vf = c.compress(torch.from_numpy(K)[None], torch.from_numpy(V)[None], torch.from_numpy(Q)[None],
                            n_rep=n_rep)
        dbg = {k: v for k, v in c.last_debug.items()}
        idx = np.asarray(dbg.get("retained_block_idx", [[]])[0] if dbg.get("retained_block_idx") else [], np.int64)
        dbg.pop("retained_block_idx", None)
        np.savez_compressed(HERE / f"compress_{name}.npz", retained_block_idx=idx,
                            k_final_sha=checksum(Kf[0].numpy()), v_final_sha=checksum(Vf[0].numpy()),
                            k_final_len=int(Kf.shape[2]), debug=json.dumps(dbg),
                            inputs_sha=checksum(K, V, Q), params=json.dumps(spec["params"]), hot=hot)
        print("compress", name, len(idx), Kf.shape)


PER_HEAD_CASES = ("ratio_l4100", "hot_l8192")


def gen_compress_per_head():
    """Per-KV-head selection keeps, for KV head h, the blocks that the reference's
    own BlockAlignedSnapKV.compress keeps when it is given that head alone: K/V
    head h with the n_rep query heads of its group (repeat_kv maps q-head i to
    kv-head i // n_rep, core/compress.py:7-20), so the block score is the max over
    that group's heads only.  One reference call per head."""
    from compress import BlockAlignedSnapKV
    for name in PER_HEAD_CASES:
        spec = COMPRESS_CASES[name]
        K, V, Q, _ = compress_case(**spec["case"])
        n_rep = spec["case"]["n_rep"]
        idx, k_sha, v_sha, lens = [], [], [], []
        for h in range(K.shape[0]):
            c = BlockAlignedSnapKV(**spec["params"])
            Kf, Vf = c.compress(torch.from_numpy(K[h:h + 1])[None], torch.from_numpy(V[h:h + 1])[None],
                                torch.from_numpy(Q[h * n_rep:(h + 1) * n_rep])[None], n_rep=n_rep)
            idx.append(np.asarray(c.last_debug["retained_block_idx"][0], np.int64))
            k_sha.append(checksum(Kf[0].numpy()))
            v_sha.append(checksum(Vf[0].numpy()))
            lens.append(int(Kf.shape[2]))
        np.savez_compressed(HERE / f"compress_perhead_{name}.npz", retained_block_idx=np.stack(idx),
                            k_final_sha=np.asarray(k_sha), v_final_sha=np.asarray(v_sha),
                            k_final_len=np.asarray(lens), inputs_sha=checksum(K, V, Q),
                            params=json.dumps(spec["params"]))
        print("compress_perhead", name, np.stack(idx).shape)


class _CpuTorch(types.ModuleType):
    """Proxy of the torch module that maps every 'cuda' device to the CPU."""

    def __init__(self):
        super().__init__("torch")

    def __getattr__(self, name):
        attr = getattr(torch, name)
        if name == "device":
            return lambda *a, **k: torch.device("cpu")
        if name in ("tensor", "zeros", "empty", "arange", "ones"):
            def wrap(*a, **k):
                if "device" in k:
                    k["device"] = "cpu"
                return attr(*a, **k)
            return wrap
        return attr


def _fake_scheduler(sink, obs, budget=0, ratio=0.2, n_rep=4, head_dim=128, pool=None, num_layers=1):
    import scheduler as sched_mod
    from compress import BlockAlignedSnapKV
    s = object.__new__(sched_mod.KVScheduler)
    s.snapkv = BlockAlignedSnapKV(16, sink, obs, ratio, budget)
    s.snapkv_anchor_tokens = max(0, int(min(16, obs)))
    s.n_rep = n_rep
    s.head_dim = head_dim
    s.num_layers = num_layers
    s.pool = pool
    return s


def gen_scores():
    import scheduler as sched_mod
    real = sched_mod.torch
    sched_mod.torch = _CpuTorch()
    try:
        for name, spec in {"l2795_d32": dict(seed=7, h_kv=8, L=2795, d=32, n_rep=4, window=16, sink=16, obs=16),
                           "l4100_d64": dict(seed=11, h_kv=8, L=4100, d=64, n_rep=4, window=64, sink=64, obs=64)}.items():
            K, V, Q, _ = compress_case(seed=spec["seed"], h_kv=spec["h_kv"], L=spec["L"], d=spec["d"],
                                       n_rep=spec["n_rep"], window=spec["window"])
            s = _fake_scheduler(spec["sink"], spec["obs"], n_rep=spec["n_rep"], head_dim=spec["d"])
            score = sched_mod.KVScheduler._score_layer_blocks_for_selection(s, torch.from_numpy(K), torch.from_numpy(Q))
            np.savez_compressed(HERE / f"score_{name}.npz", score=score.numpy(), inputs_sha=checksum(K, V, Q),
                                spec=json.dumps(spec))
            print("score", name, score.shape)
    finally:
        sched_mod.torch = real


def gen_budget():
    rows = []
    for sink, obs, budget, ratio in [(16, 16, 2048, 0.2), (64, 64, 0, 0.2), (64, 64, 0, 0.25), (16, 16, 0, 0.01),
                                     (64, 128, 0, 0.25), (16, 16, 512, 0.2)]:
        s = _fake_scheduler(sink, obs, budget=budget, ratio=ratio)
        import scheduler as sched_mod
        for L in [10, 47, 48, 49, 95, 96, 500, 511, 512, 513, 600, 2048, 2049, 2795, 4100, 16500, 32768, 131072]:
            k, eff, mode = sched_mod.KVScheduler._selection_budget_blocks(s, L)
            rows.append(dict(sink=sink, obs=obs, budget=budget, ratio=ratio, L=L, k=k, eff=eff, mode=mode))
    (HERE / "budget.json").write_text(json.dumps(rows, indent=0))
    print("budget", len(rows))


class _CpuPool:
    def __init__(self, n_pages, h_kv, d, dtype):
        self.B = 16
        self.dtype = dtype
        self.k_cache = torch.full((1, n_pages, 16, h_kv, d), -7.0, dtype=dtype)
        self.v_cache = torch.full((1, n_pages, 16, h_kv, d), -9.0, dtype=dtype)


def gen_writeback():
    import scheduler as sched_mod
    real_to = torch.Tensor.to

    def to_cpu(self, *a, **k):
        a = tuple("cpu" if x == "cuda" else x for x in a)
        if k.get("device") == "cuda":
            k["device"] = "cpu"
        return real_to(self, *a, **k)

    real = sched_mod.torch
    sched_mod.torch = _CpuTorch()
    torch.Tensor.to = to_cpu
    try:
        cases = {
            # aligned fast path (sink, obs, L multiples of 16)
            "aligned": dict(seed=21, h_kv=2, L=512, d=16, sink=32, obs=32, k=6),
            # unaligned L: piecewise path with zero padding of the last mid block
            "unaligned": dict(seed=22, h_kv=2, L=509, d=16, sink=16, obs=16, k=5),
            # unaligned sink/obs lengths
            "odd_sink": dict(seed=23, h_kv=3, L=300, d=8, sink=5, obs=7, k=4),
        }
        for name, c in cases.items():
            rng = np.random.default_rng(c["seed"])
            K = rng.standard_normal((c["h_kv"], c["L"], c["d"])).astype(np.float32)
            V = rng.standard_normal((c["h_kv"], c["L"], c["d"])).astype(np.float32)
            n_mid = -(-(c["L"] - c["sink"] - c["obs"]) // 16)
            sel = np.sort(rng.choice(n_mid, size=c["k"], replace=False)).astype(np.int64)
            # always include the last (possibly partial) mid block
            sel[-1] = n_mid - 1
            sel = np.unique(sel)
            eff = c["sink"] + 16 * len(sel) + c["obs"]
            n_dst = -(-eff // 16)
            pool = _CpuPool(n_dst + 8, c["h_kv"], c["d"], torch.float32)
            dst = [int(x) for x in rng.permutation(n_dst + 8)[:n_dst]]
            s = _fake_scheduler(c["sink"], c["obs"], pool=pool)
            sched_mod.KVScheduler._write_selected_layer_to_pool(
                s, 0, dst, torch.from_numpy(K), torch.from_numpy(V), [int(x) for x in sel], eff, "ratio")
            np.savez_compressed(HERE / f"writeback_{name}.npz", K=K, V=V, selected=sel, dst=np.asarray(dst, np.int32),
                                eff=eff, sink=c["sink"], obs=c["obs"], n_pool=n_dst + 8,
                                k_pool=pool.k_cache[0].numpy(), v_pool=pool.v_cache[0].numpy())
            print("writeback", name, eff, n_dst)
    finally:
        sched_mod.torch = real
        torch.Tensor.to = real_to


if __name__ == "__main__":
    which = set(sys.argv[1:]) or {"page16", "compress", "perhead", "score", "budget", "writeback"}
    if "page16" in which:
        gen_page16()
    if "compress" in which:
        gen_compress()
    if "perhead" in which:
        gen_compress_per_head()
    if "score" in which:
        gen_scores()
    if "budget" in which:
        gen_budget()
    if "writeback" in which:
        gen_writeback()
