"""CPU tests of the chunked-prefill host loop (core/chunked_prefill.py:5-39):
chunk boundaries, the past cache threaded through the calls, the last
position's logits, and the memory estimate."""
import torch

from unifiedkv_b200.chunked_prefill import ChunkedPrefillProcessor


class _Out:
    def __init__(self, logits, past):
        self.logits, self.past_key_values = logits, past


class _FakeModel:
    """Records each call; logits = token ids, the 'cache' = every id seen so far."""

    def __init__(self):
        self.calls = []

    def __call__(self, input_ids, past_key_values, use_cache):
        assert use_cache
        self.calls.append((input_ids.clone(), past_key_values))
        seen = input_ids if past_key_values is None else torch.cat([past_key_values, input_ids], dim=1)
        return _Out(input_ids.float()[..., None].repeat(1, 1, 3), seen)


def test_chunk_loop_threads_the_cache():
    ids = torch.arange(10)[None]
    m = _FakeModel()
    logits, past = ChunkedPrefillProcessor(chunk_size=4).run(m, ids)
    assert [c[0].tolist() for c in m.calls] == [[[0, 1, 2, 3]], [[4, 5, 6, 7]], [[8, 9]]]
    assert m.calls[0][1] is None and torch.equal(m.calls[2][1], ids[:, :8])
    assert logits.shape == (1, 1, 3) and torch.all(logits == 9)
    assert torch.equal(past, ids)
    m2 = _FakeModel()
    ChunkedPrefillProcessor(chunk_size=4).run(m2, ids, chunk_size=16)  # the per-call size wins
    assert len(m2.calls) == 1


def test_estimate_peak_gb():
    full, chunk = ChunkedPrefillProcessor.estimate_peak_gb(32768, 32, 128, 2048)
    assert full == 32 * 32768 * 32768 * 2 / 1024 ** 3 and chunk == 32 * 2048 * 32768 * 2 / 1024 ** 3
