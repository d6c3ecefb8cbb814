"""GPU parity of the Page16 decode kernel (libbpkv.so) against the oracle.

Tolerances (from the spec of this path): fp32 inputs max-abs 1e-5 against an
fp64 restatement; bf16 / fp16 inputs max-abs 2e-3 against the fp32/fp64
restatement of the same (rounded) inputs.
"""
import math

import numpy as np
import pytest
import torch

from oracle.page16 import page16_decode_reference
from tests.golden.inputs import PAGE16_CASES, page16_case

pytestmark = pytest.mark.gpu
GOLDEN = __import__("pathlib").Path(__file__).parent / "golden"
TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3}


def _err(out, ref, dtype):
    """Max-abs error beyond the output format's own rounding.

    The output has q's dtype (as in the reference, empty_like(q)); storing a value
    x in bf16 / fp16 alone costs up to |x| * 2^-8 / 2^-11, so the 2e-3 budget
    bounds the arithmetic error on top of that unavoidable rounding.
    """
    ref = np.asarray(ref, np.float64)
    fmt = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}.get(dtype, 0.0)
    return float(np.nanmax(np.abs(out - ref) - fmt * np.abs(ref)))


def _run(cuda, q, k, v, bt, lens, dtype, scale=None, lse=False, layer_view=False):
    from unifiedkv_b200.page16_native import page16_decode_attention
    d = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    tq = torch.from_numpy(np.asarray(q, np.float32)).to(cuda, dtype)
    tk = torch.from_numpy(np.asarray(k, np.float32)).to(cuda, dtype)
    tv = torch.from_numpy(np.asarray(v, np.float32)).to(cuda, dtype)
    if layer_view:  # exercise a non-zero layer of a [L, N, 16, h, d] pool
        pool_k = torch.zeros((3,) + tuple(tk.shape), dtype=dtype, device=cuda)
        pool_v = torch.zeros_like(pool_k)
        pool_k[1].copy_(tk)
        pool_v[1].copy_(tv)
        tk, tv = pool_k[1], pool_v[1]
    lse_t = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=cuda) if lse else None
    out = page16_decode_attention(tq, tk, tv, torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda),
                                  softmax_scale=scale, n_rep=q.shape[1] // k.shape[2], lse_out=lse_t)
    torch.cuda.synchronize()
    # oracle sees exactly the rounded inputs the kernel saw
    qr, kr, vr = (t.float().cpu().numpy() for t in (tq, tk, tv))
    return out.float().cpu().numpy(), (lse_t.cpu().numpy() if lse else None), (qr, kr, vr)


@pytest.mark.parametrize("name", sorted(PAGE16_CASES))
def test_golden_cases(cuda, name):
    cfg = PAGE16_CASES[name]
    q, k, v, bt, lens = page16_case(**cfg)
    dtype = torch.float32 if q.dtype == np.float32 else torch.float16
    out, _, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, dtype)
    g = np.load(GOLDEN / f"page16_{name}.npz")
    ref = page16_decode_reference(qr, kr, vr, bt, lens, float(g["scale"]), int(g["n_rep"]))
    assert _err(out, ref, dtype) < TOL[dtype]
    # and against the reference kernel's own output
    assert np.max(np.abs(out - g["out"])) < (1e-5 if dtype == torch.float32 else 2e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (8, 2, 64), (16, 1, 128), (8, 8, 128), (8, 4, 256),
                                      (12, 3, 96), (40, 2, 64)])
def test_shapes_and_dtypes(cuda, dtype, hq, hkv, d):
    lens = (1, 15, 16, 17, 129, 700, 2049)
    q, k, v, bt, lens = page16_case(seed=hq * 7 + d, batch=len(lens), hq=hq, hkv=hkv, d=d, lens=lens,
                                    num_pages=300, scale_std=0.5)
    out, lse, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, dtype, lse=True)
    ref, ref_lse = page16_decode_reference(qr, kr, vr, bt, lens, 1 / math.sqrt(d), hq // hkv, return_lse=True)
    assert _err(out, ref, dtype) < TOL[dtype]
    assert np.max(np.abs(lse - ref_lse)) < 1e-3


def test_empty_and_capped_lengths(cuda):
    # len 0 -> NaN row (reference 0/0); len beyond 16*max_blocks reads max_blocks pages only
    q, k, v, bt, lens = page16_case(seed=31, batch=4, hq=8, hkv=2, d=128, lens=(0, 40, 1000, 3),
                                    num_pages=100, max_blocks=20, scale_std=0.5)
    out, _, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, torch.bfloat16)
    ref = page16_decode_reference(qr, kr, vr, bt, lens, 1 / math.sqrt(128), 4)
    assert np.isnan(out[0]).all()
    assert np.isfinite(out[1:]).all()
    assert _err(out[1:], ref[1:], torch.bfloat16) < 2e-3


def test_layer_view_and_stale_pages(cuda):
    # pages past len hold NaN: must not leak into the output (reference masks them)
    q, k, v, bt, lens = page16_case(seed=32, batch=3, hq=16, hkv=4, d=128, lens=(33, 250, 17),
                                    num_pages=64, scale_std=0.5)
    k = k.copy(); v = v.copy()
    for b, l in enumerate(lens):
        last = bt[b, (l - 1) // 16]
        k[last, l % 16 or 16:] = np.nan
        v[last, l % 16 or 16:] = np.nan
    out, _, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, torch.bfloat16, layer_view=True)
    ref = page16_decode_reference(qr, kr, vr, bt, lens, 1 / math.sqrt(128), 4)
    assert np.isfinite(out).all()
    assert _err(out, ref, torch.bfloat16) < 2e-3


def test_llama8b_decode_layer_sampled(cuda):
    """Config 2 shapes (one layer): B=32, 32/8 heads, d=128, ctx U[4096,32768], bf16, q/k/v ~ 0.5 N(0,1)."""
    from unifiedkv_b200.page16_native import page16_decode_attention
    rng = np.random.default_rng(2)
    B, hq, hkv, d = 32, 32, 8, 128
    lens = rng.integers(4096, 32769, size=B).astype(np.int32)
    need = (lens + 15) // 16
    n_pages = int(need.sum()) + 64
    g = torch.Generator(device=cuda).manual_seed(2)
    kc = (torch.randn((n_pages, 16, hkv, d), generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    vc = (torch.randn((n_pages, 16, hkv, d), generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    q = (torch.randn((B, hq, d), generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    perm = rng.permutation(n_pages).astype(np.int32)
    mb = int(need.max())
    bt = np.zeros((B, mb), np.int32)
    off = 0
    for b in range(B):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += need[b]
    out = page16_decode_attention(q, kc, vc, torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda),
                                  softmax_scale=d ** -0.5, n_rep=4)
    out2 = page16_decode_attention(q, kc, vc, torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda),
                                   softmax_scale=d ** -0.5, n_rep=4)
    torch.cuda.synchronize()
    assert torch.equal(out, out2), "decode must be deterministic"
    for b in [0, 7, 19, 31]:
        ids = torch.from_numpy(bt[b, :need[b]].astype(np.int64)).to(cuda)
        kb = kc.index_select(0, ids).float().cpu().numpy()
        vb = vc.index_select(0, ids).float().cpu().numpy()
        ref = page16_decode_reference(q[b:b + 1].float().cpu().numpy(), kb, vb,
                                      np.arange(need[b], dtype=np.int32)[None], lens[b:b + 1], d ** -0.5, 4,
                                      compute_dtype=np.float32)
        assert _err(out[b:b + 1].float().cpu().numpy(), ref, torch.bfloat16) < 2e-3


def test_single_sequence_131k(cuda):
    """Config 3 shapes: one request of 131072 tokens (8192 pages), 32/8 heads, bf16."""
    from unifiedkv_b200.page16_native import page16_decode_attention
    d, hq, hkv, L = 128, 32, 8, 131072
    g = torch.Generator(device=cuda).manual_seed(3)
    n_pages = L // 16
    kc = torch.randn((n_pages, 16, hkv, d), generator=g, device=cuda).to(torch.bfloat16)
    vc = torch.randn((n_pages, 16, hkv, d), generator=g, device=cuda).to(torch.bfloat16)
    q = (torch.randn((1, hq, d), generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    bt = torch.randperm(n_pages, generator=g, device=cuda).to(torch.int32)[None]
    lens = torch.tensor([L], dtype=torch.int32, device=cuda)
    out = page16_decode_attention(q, kc, vc, bt, lens, softmax_scale=d ** -0.5, n_rep=4)
    ids = bt[0].long()
    ref = page16_decode_reference(q.float().cpu().numpy(), kc.index_select(0, ids).float().cpu().numpy(),
                                  vc.index_select(0, ids).float().cpu().numpy(),
                                  np.arange(n_pages, dtype=np.int32)[None], np.array([L], np.int32), d ** -0.5, 4,
                                  compute_dtype=np.float32)
    assert _err(out.float().cpu().numpy(), ref, torch.bfloat16) < 2e-3


def test_decode_append_then_decode(cuda):
    from unifiedkv_b200.page16_native import decode_append
    q, k, v, bt, lens = page16_case(seed=40, batch=3, hq=8, hkv=2, d=64, lens=(15, 16, 40), num_pages=20,
                                    max_blocks=4, scale_std=0.5)
    tk = torch.from_numpy(k).to(cuda, torch.bfloat16)
    tv = torch.from_numpy(v).to(cuda, torch.bfloat16)
    knew = torch.randn(3, 2, 64, device=cuda).to(torch.bfloat16)
    vnew = torch.randn(3, 2, 64, device=cuda).to(torch.bfloat16)
    tbt = torch.from_numpy(bt).to(cuda)
    decode_append(knew, vnew, tk, tv, tbt, torch.from_numpy(lens).to(cuda))
    torch.cuda.synchronize()
    for b, l in enumerate(lens):
        page = bt[b, l // 16]
        assert torch.equal(tk[page, l % 16], knew[b]) and torch.equal(tv[page, l % 16], vnew[b])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_fused_append_matches_append_then_decode(cuda, dtype, d):
    """The append fused into the decode launch gives bit-identical outputs and pool
    contents to decode_append followed by page16_decode_attention (lengths that
    end on a page boundary, a 1-token request, an empty one, one past the
    block-table capacity, and long ones split across CTAs)."""
    from unifiedkv_b200.page16_native import decode_append, page16_decode_attention
    lens = (1, 16, 17, 0, 70, 2000, 4096)
    hq, hkv, max_blocks = 8, 2, 256
    q, k, v, bt, lens = page16_case(seed=41 + d, batch=len(lens), hq=hq, hkv=hkv, d=d, lens=lens,
                                    num_pages=2048, max_blocks=max_blocks, scale_std=0.5)
    lens = lens.copy()
    lens[-1] = max_blocks * 16 + 5  # beyond the table: decoded capped, nothing appended
    g = torch.Generator(device="cpu").manual_seed(7)
    knew = torch.randn(len(lens), hkv, d, generator=g).to(cuda, dtype)
    vnew = torch.randn(len(lens), hkv, d, generator=g).to(cuda, dtype)
    tq = torch.from_numpy(q).to(cuda, dtype)
    tbt = torch.from_numpy(bt).to(cuda)
    tl = torch.from_numpy(lens).to(cuda)
    k0 = torch.from_numpy(k).to(cuda, dtype)
    v0 = torch.from_numpy(v).to(cuda, dtype)
    ka, va = k0.clone(), v0.clone()
    decode_append(knew, vnew, ka, va, tbt, (tl - 1).clamp(min=-1))
    lse_a = torch.empty(len(lens), hq, device=cuda)
    out_a = page16_decode_attention(tq, ka, va, tbt, tl, softmax_scale=d ** -0.5, n_rep=hq // hkv, lse_out=lse_a)
    kf, vf = k0.clone(), v0.clone()
    lse_f = torch.empty(len(lens), hq, device=cuda)
    out_f = page16_decode_attention(tq, kf, vf, tbt, tl, softmax_scale=d ** -0.5, n_rep=hq // hkv,
                                    lse_out=lse_f, k_new=knew, v_new=vnew)
    torch.cuda.synchronize()
    assert torch.equal(kf, ka) and torch.equal(vf, va)
    # the empty request's row is NaN on both paths (0/0, as in the reference)
    torch.testing.assert_close(out_f, out_a, rtol=0, atol=0, equal_nan=True)
    torch.testing.assert_close(lse_f, lse_a, rtol=0, atol=0, equal_nan=True)


def test_shape_errors_use_reference_tokens(cuda):
    from unifiedkv_b200.page16_native import page16_decode_attention
    q = torch.zeros(2, 6, 64, device=cuda, dtype=torch.bfloat16)
    kc = torch.zeros(4, 16, 4, 64, device=cuda, dtype=torch.bfloat16)
    bt = torch.zeros(2, 2, dtype=torch.int32, device=cuda)
    lens = torch.ones(2, dtype=torch.int32, device=cuda)
    with pytest.raises(RuntimeError, match="page16_native_shape_unsupported:gqa"):
        page16_decode_attention(q, kc, kc, bt, lens, softmax_scale=0.1, n_rep=1)
    with pytest.raises(RuntimeError, match="page16_native_shape_unsupported:block_size_8"):
        page16_decode_attention(q, kc[:, :8], kc[:, :8], bt, lens, softmax_scale=0.1, n_rep=1)
    with pytest.raises(RuntimeError, match="page16_native_shape_unsupported:block_table_batch"):
        page16_decode_attention(q[:, :4], kc, kc, bt[:1], lens, softmax_scale=0.1, n_rep=1)


def test_decode_large_logits(cuda):
    """Logits of several hundred (natural log units) with keys growing along the
    sequence: the running max keeps moving and exp underflows for most keys."""
    q, k, v, bt, lens = page16_case(seed=61, batch=3, hq=32, hkv=8, d=128, lens=(5000, 37, 900), num_pages=400,
                                    scale_std=1.0)
    ramp = np.linspace(0.2, 6.0, 16 * 400, dtype=np.float32).reshape(400, 16, 1, 1)
    k = (k * ramp).astype(np.float32)
    q = (q * 8.0).astype(np.float32)
    out, _, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, torch.bfloat16)
    ref = page16_decode_reference(qr, kr, vr, bt, lens, 1 / math.sqrt(128), 4)
    assert np.isfinite(out).all()
    assert _err(out, ref, torch.bfloat16) < 2e-3


@pytest.mark.parametrize("hkv,d", [(8, 128), (8, 64), (4, 256)])
def test_single_request_split_over_ctas(cuda, hkv, d):
    """Batch 1 (one long request split over every CTA, merged by the combine kernel).
    Lengths from empty (NaN row, lse -inf) through fewer pages than CTAs (empty CTA
    ranges) to many pages per CTA; every length twice in a row, with lse_out."""
    hq = 4 * hkv
    for L in (0, 1, 17, 100 * 16 + 3, 147 * 16, 148 * 16 + 1, 5000, 40000):
        for rep in range(2):
            q, k, v, bt, lens = page16_case(seed=L + rep, batch=1, hq=hq, hkv=hkv, d=d, lens=(L,),
                                            num_pages=max(4, (L + 15) // 16 + 3), scale_std=0.5)
            out, lse, (qr, kr, vr) = _run(cuda, q, k, v, bt, lens, torch.bfloat16, lse=True)
            if L == 0:
                assert np.isnan(out).all() and np.isneginf(lse).all()
                continue
            ref, ref_lse = page16_decode_reference(qr, kr, vr, bt, lens, 1.0 / math.sqrt(d), 4, return_lse=True)
            assert _err(out, ref, torch.bfloat16) < 2e-3, (L, rep)
            assert np.abs(lse - ref_lse).max() < 1e-3, (L, rep)


def test_single_request_graph_replay(cuda):
    """The batch-1 decode captured in a CUDA graph and replayed with new lengths
    (the grid split and the combine follow the lengths on the device)."""
    from unifiedkv_b200.page16_native import page16_decode_attention
    q, k, v, bt, lens = page16_case(seed=3, batch=1, hq=32, hkv=8, d=128, lens=(30000,), num_pages=1900,
                                    scale_std=0.5)
    tq, tk, tv = (torch.from_numpy(x).to(cuda, torch.bfloat16) for x in (q, k, v))
    tbt = torch.from_numpy(bt).to(cuda)
    tl = torch.from_numpy(lens).to(cuda)
    page16_decode_attention(tq, tk, tv, tbt, tl, softmax_scale=128 ** -0.5, n_rep=4)  # warm (workspace)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = page16_decode_attention(tq, tk, tv, tbt, tl, softmax_scale=128 ** -0.5, n_rep=4)
    qr, kr, vr = (t.float().cpu().numpy() for t in (tq, tk, tv))
    for L in (30000, 9, 2371, 30000):
        tl.fill_(L)
        g.replay()
        torch.cuda.synchronize()
        ref = page16_decode_reference(qr, kr, vr, bt, np.array([L], np.int32), 128 ** -0.5, 4)
        assert _err(out.float().cpu().numpy(), ref, torch.bfloat16) < 2e-3, L
