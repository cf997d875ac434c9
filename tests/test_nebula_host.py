"""Nebula host logic on the CPU (reference tests/test_nebula_cache.py and
tests/test_nebula_runtime.py semantics): KV-cache bookkeeping, model config
and init, the engine protocol, validation and failure poisoning.  The engine
runs with the CPU sharded decoder harness; the product decoder itself is
CUDA-only and refuses a CPU context."""

import pytest
import torch

from forgeml_b200.nebula import (CacheError, DecoderConfig, Engine, EngineFailed, KVCache, ParallelContext,
                                 ShardedDecoder, TinyDecoder)
from tests.cpu_engine import CpuShardedDecoder
from tests.golden_io import load_nebula_small


def cache(**kw):
    args = dict(layer_ids=(0, 1), num_heads=2, head_dim=4, max_seq_len=8, max_requests=4,
                device=torch.device("cpu"), dtype=torch.float32)
    args.update(kw)
    return KVCache(**args)


def kv(b, t, v=1.0):
    return torch.full((b, 2, t, 4), v)


def test_cache_append_returns_prefix():
    c = cache()
    c.reserve((7, 9))
    k0, _ = c.append(0, (7, 9), kv(2, 3, 1.0), kv(2, 3, 2.0), 0)
    assert k0.shape == (2, 2, 3, 4)
    c.append(1, (7, 9), kv(2, 3), kv(2, 3), 0)
    k1, v1 = c.append(0, (7, 9), kv(2, 1, 5.0), kv(2, 1, 6.0), 3)
    assert k1.shape == (2, 2, 4, 4)
    assert (k1[:, :, :3] == 1.0).all() and (k1[:, :, 3] == 5.0).all() and (v1[:, :, 3] == 6.0).all()


def test_cache_reserve_rejects_without_mutation():
    c = cache(max_requests=2)
    with pytest.raises(CacheError):
        c.reserve((1, 1))
    assert c.active_requests == 0
    c.reserve((1, 2))
    with pytest.raises(CacheError):
        c.reserve((3, 4))
    assert c.active_requests == 2
    with pytest.raises(CacheError):
        c.reserve((1,))


def test_cache_append_validation():
    c = cache()
    c.reserve((5,))
    for args in (((5, 5), kv(2, 1), kv(2, 1), 0), ((5,), kv(2, 1), kv(2, 1), 1), ((5,), kv(1, 9), kv(1, 9), 0),
                 ((5,), kv(1, 1), kv(1, 2), 0), ((99,), kv(1, 1), kv(1, 1), 0)):
        with pytest.raises(CacheError):
            c.append(0, *args)
    with pytest.raises(CacheError):
        c.append(2, (5,), kv(1, 1), kv(1, 1), 0)
    c.append(0, (5,), kv(1, 2), kv(1, 2), 0)
    with pytest.raises(CacheError):
        c.append(0, (5,), kv(1, 1), kv(1, 1), 0)
    with pytest.raises(CacheError):
        c.append(0, (5,), kv(1, 7), kv(1, 7), 2)
    k, _ = c.append(1, (5,), kv(1, 2, 3.0), kv(1, 2), 0)
    assert k.shape == (1, 2, 2, 4)


def test_cache_release_reuse_and_slots():
    c = cache(max_requests=2)
    c.reserve((3,))
    c.reserve((4,))
    assert c.slots((3, 4)) == [0, 1]
    c.release((3,))
    c.release((3,))
    assert c.active_requests == 1
    c.reserve((8,))
    assert c.slots((8,)) == [0]  # lowest free slot is reused
    c.clear()
    assert c.active_requests == 0
    # a request's slot block has the reference's per-request layout [heads, max_seq, hd]
    c.reserve((1,))
    assert c.k_pool[0][c.slots((1,))[0]].shape == (2, 8, 4)


def test_cache_validate_positions():
    c = cache()
    c.reserve((1,))
    c.validate((1,), 0, 2)
    c.append(0, (1,), kv(1, 2), kv(1, 2), 0)
    with pytest.raises(CacheError):
        c.validate((1,), 2, 1)
    c.append(1, (1,), kv(1, 2), kv(1, 2), 0)
    c.validate((1,), 2, 1)


def test_config_validation_and_reference_init():
    with pytest.raises(ValueError):
        DecoderConfig(hidden_size=10, num_heads=3)
    with pytest.raises(ValueError):
        DecoderConfig(vocab_size=0)
    gold = load_nebula_small()
    sd = TinyDecoder(DecoderConfig(**gold["config"])).state_dict()
    assert all(torch.equal(sd[k], v) for k, v in gold["state_dict"].items())


def cfg():
    return DecoderConfig(**load_nebula_small()["config"])


def engine(**kw):
    return Engine(cfg(), context=ParallelContext.from_env(), max_requests=4, decoder_factory=CpuShardedDecoder, **kw)


def test_product_decoder_refuses_cpu():
    with pytest.raises(ValueError, match="CUDA"):
        ShardedDecoder(cfg(), ParallelContext.from_env())


def test_engine_protocol_matches_reference_outputs():
    gold = load_nebula_small()
    e = engine()
    got = e.forward(gold["prefill_tokens"], gold["prefill_ids"], 0)
    torch.testing.assert_close(got, gold["prefill_logits"], rtol=1e-5, atol=1e-6)
    got_d = e.forward(gold["decode_tokens"], gold["prefill_ids"], 3)
    torch.testing.assert_close(got_d, gold["decode_logits"], rtol=1e-5, atol=1e-6)
    e.release(gold["prefill_ids"])
    assert e.generate(gold["generate_prompts"], 3) == gold["generate_tokens"]
    assert e.decoder.cache.active_requests == 0
    assert e.generate([[1, 2]], 0) == [[]]
    prompts = gold["generate_prompts"] + [[3, 1, 4, 1, 5]]
    want = [e.generate([p], 3)[0] for p in prompts]
    assert e.generate_mixed(prompts, 3) == want
    assert e.decoder.cache.active_requests == 0
    e.close()


def test_invalid_requests_do_not_poison():
    e = engine()
    for toks, ids, pos in ((torch.tensor([[1, 2]]), (1,), 15), (torch.tensor([[1, 99]]), (1,), 0),
                           (torch.tensor([[1]]), (1, 2), 0), (torch.tensor([[1]]), (1 << 62,), 0)):
        with pytest.raises(ValueError):
            e.forward(toks, ids, pos)
    with pytest.raises(TypeError):
        e.forward(torch.tensor([[1]]), (1,), 0.0)
    assert e.healthy
    assert e.forward(torch.tensor([[1, 2]]), (3,), 0).shape == (1, 2, 32)
    e.close()


@pytest.mark.parametrize("failure", [RuntimeError, KeyError, AssertionError])
def test_failed_forward_poisons_engine(monkeypatch, failure):
    e = engine()
    e.forward(torch.tensor([[1, 2]]), (8,), 0)

    def boom(*a, **k):
        raise failure("simulated failure")

    monkeypatch.setattr(e.decoder, "forward", boom)
    with pytest.raises(EngineFailed):
        e.forward(torch.tensor([[3]]), (8,), 2)
    assert not e.healthy and e.decoder.cache.active_requests == 0
    with pytest.raises(EngineFailed):
        e.forward(torch.tensor([[1]]), (9,), 0)
    e.close()


def test_broadcast_failure_poisons_and_close_skips(monkeypatch):
    e = engine()
    sent = []

    def dead_transport(t):
        sent.append(t.clone())
        raise RuntimeError("transport dead")

    monkeypatch.setattr(e, "_multi", True)
    monkeypatch.setattr(e._wire, "broadcast", dead_transport)
    with pytest.raises(EngineFailed):
        e.forward(torch.tensor([[5]]), (1,), 0)
    assert not e.healthy and e.decoder.cache.active_requests == 0
    e.close()  # an unhealthy leader sends no STOP
    assert len(sent) == 1
    # the frame that failed to go out: the reference's int64 STEP header, then
    # the request id and the token, zero padded to 4 + 2 * max_requests words
    frame = sent[0]
    assert frame.dtype == torch.int64 and frame.numel() == 4 + 3 * 4
    assert frame.tolist() == [1, 1, 1, 0, 1, 5] + [0] * 10


def test_wire_frames_split_when_the_message_is_long():
    from forgeml_b200.nebula.engine import CMD_STEP, _CommandWire

    w = _CommandWire(max_requests=2, max_seq_len=16, device=torch.device("cpu"))
    sent = []
    w.broadcast = lambda t: sent.append(t.clone())
    w.send(CMD_STEP, 0, (7, 9), torch.tensor([[1, 2, 3], [4, 5, 6]]))
    assert [t.tolist() for t in sent] == [[1, 2, 3, 0] + [0] * 6, [7, 9, 1, 2, 3, 4, 5, 6]]
    # the receiving side rebuilds the same command from the same words
    frames = iter(sent)
    r = _CommandWire(max_requests=2, max_seq_len=16, device=torch.device("cpu"))
    r.broadcast = lambda t: t.copy_(next(frames))
    c = r.receive()
    assert (c.cmd, c.batch, c.steps, c.start, c.ids) == (1, 2, 3, 0, (7, 9))
    assert c.tokens.tolist() == [[1, 2, 3], [4, 5, 6]]


@pytest.mark.parametrize("max_requests", [4, 2])
def test_wire_prefill_batches_round_trip(max_requests):
    """CMD_PREFILL: groups of equal-length prompts in one command (in the
    fixed frame when they fit, else header frame + body), rebuilt word for
    word on the receiving side."""
    from forgeml_b200.nebula.engine import CMD_PREFILL, _CommandWire

    groups = [((11,), torch.tensor([[1, 2, 3]])), ((12, 13), torch.tensor([[4, 5], [6, 7]]))]
    if max_requests == 2:  # 3 ids do not fit a 2-request engine's admission, so use smaller groups
        groups = [((11,), torch.tensor([[1, 2, 3, 4, 5, 6, 7]])), ((12,), torch.tensor([[8, 9]]))]
    w = _CommandWire(max_requests=max_requests, max_seq_len=16, device=torch.device("cpu"))
    sent = []
    w.broadcast = lambda t: sent.append(t.clone())
    w.send_prefill(groups)
    body = [v for ids, tok in groups for v in (len(ids), tok.shape[1])] + [r for ids, _ in groups for r in ids]
    body += [x for _, tok in groups for x in tok.reshape(-1).tolist()]
    head = [CMD_PREFILL, len(groups), len(body), 0]
    if 4 + len(body) <= w.frame_words:
        assert [t.tolist() for t in sent] == [head + body + [0] * (w.frame_words - 4 - len(body))]
    else:
        assert [t.tolist() for t in sent] == [head + [0] * (w.frame_words - 4), body]
    frames = iter(sent)
    r = _CommandWire(max_requests=max_requests, max_seq_len=16, device=torch.device("cpu"))
    r.broadcast = lambda t: t.copy_(next(frames))
    c = r.receive()
    assert c.cmd == CMD_PREFILL and len(c.groups) == len(groups)
    for (ids, tok), (gids, gtok) in zip(groups, c.groups):
        assert tuple(gids) == ids and gtok.tolist() == tok.tolist()


def test_wire_rejects_malformed_prefill():
    from forgeml_b200.nebula.engine import _CommandWire

    # header fits, body sizes inconsistent with the word count
    for words in ([4, 1, 6, 0, 1, 2, 7, 1, 2, 3], [4, 0, 3, 0], [4, 1, 4, 1, 1, 1, 7, 1], [4, 1, 4, 0, 1, 17, 7, 1]):
        r = _CommandWire(max_requests=2, max_seq_len=16, device=torch.device("cpu"))
        r.broadcast = lambda t, words=words: t[:len(words)].copy_(torch.tensor(words))
        with pytest.raises(EngineFailed):
            r.receive()


def test_wire_rejects_malformed_headers():
    from forgeml_b200.nebula.engine import _CommandWire

    for words in ([0, 1, 0, 0], [1, 3, 1, 0], [1, 1, 0, 0], [1, 1, 2, 15], [2, 1, 1, 0], [7, 0, 0, 0]):
        r = _CommandWire(max_requests=2, max_seq_len=16, device=torch.device("cpu"))
        r.broadcast = lambda t, words=words: t[:4].copy_(torch.tensor(words))
        with pytest.raises(EngineFailed):
            r.receive()


def test_closed_engine_and_release_checks():
    e = engine()
    with pytest.raises(ValueError):
        e.release((1 << 63,))
    assert e.healthy
    e.forward(torch.tensor([[1, 2]]), (1,), 0)
    e.release((1,))
    assert e.decoder.cache.active_requests == 0
    e.close()
    with pytest.raises(EngineFailed):
        e.forward(torch.tensor([[1]]), (1,), 0)
    with pytest.raises(EngineFailed):
        e.generate([[1]], 1)


def test_cache_layers_move_apart_and_back_together():
    """Per-layer counts appear while reference-style appends move one layer
    ahead of the others and merge again once they agree; the checks and their
    messages are per layer in layer order throughout."""
    c = cache(layer_ids=(3, 5, 7))
    c.reserve((1, 2))
    c.append(3, (1, 2), kv(2, 2), kv(2, 2), 0)
    with pytest.raises(CacheError, match="layer 5 for request 1 at 0, expected 2"):
        c.validate((1, 2), 2, 1)
    with pytest.raises(CacheError, match="layer 3 for request 1 at 2, expected 0"):
        c.validate((1, 2), 0, 1)
    with pytest.raises(CacheError, match="layer 3 request 1 at 2, expected 0"):
        c.append(3, (1, 2), kv(2, 2), kv(2, 2), 0)
    c.append(5, (1, 2), kv(2, 2), kv(2, 2), 0)
    c.append(7, (1, 2), kv(2, 2), kv(2, 2), 0)
    c.validate((1, 2), 2, 1)  # all three layers at 2 again
    with pytest.raises(CacheError, match="layer 3 for request 2 at 2, expected 3"):
        c.validate((2,), 3, 1)
    c.advance((1,), 5)  # the decode step: every layer of request 1 at once
    c.validate((1,), 5, 1)
    c.validate((2,), 2, 1)
    with pytest.raises(CacheError, match="layer 3 for request 1 at 5, expected 2"):
        c.validate((1, 2), 2, 1)
    c.append(7, (2,), kv(1, 1), kv(1, 1), 2)  # layer 7 ahead: others may follow
    c.advance((2,), 3)
    c.validate((2,), 3, 1)


def test_cache_id_checks_hold_for_reused_and_new_tuples():
    c = cache()
    ids = (1, 2)
    c.reserve(ids)
    c.validate(ids, 0, 1)
    c.validate(ids, 0, 1)  # the same tuple again
    for bad, msg in (((1, 1), "duplicate"), ((1, True), "invalid request id"), ((1, -1), "invalid request id"),
                     ([1, 2.0], "invalid request id"), ((), "non-empty")):
        with pytest.raises(CacheError, match=msg):
            c.validate(bad, 0, 1)
    lst = [1, 2]
    c.validate(lst, 0, 1)
    lst[1] = 1  # a list can change between calls: checked every time
    with pytest.raises(CacheError, match="duplicate"):
        c.validate(lst, 0, 1)


def test_engine_id_checks_keep_the_manual_range_for_reused_tuples():
    """A tuple accepted for an engine-internal call (ids above the manual
    range are allowed there) is checked again when a caller passes it."""
    e = engine()
    big = ((1 << 62) + 5,)
    out = e.forward(torch.tensor([[1, 2]]), big, 0, _internal=True)
    assert out.shape == (1, 2, 32)
    with pytest.raises(ValueError, match="manual range"):
        e.forward(torch.tensor([[3]]), big, 2)
    assert e.healthy
    ids = (7, 8)
    e.forward(torch.tensor([[1], [2]]), ids, 0)
    e.forward(torch.tensor([[1], [2]]), ids, 1, _internal=True)  # accepted by the stricter rules before
    e.forward(torch.tensor([[1], [2]]), ids, 2)
    assert e.healthy
    e.close()


def test_wire_returns_one_tuple_for_repeated_ids():
    """A worker receiving consecutive commands with equal ids gets the same
    tuple object back (its id checks then see a tuple they accepted);
    different ids give a new tuple."""
    from forgeml_b200.nebula.engine import CMD_RELEASE, CMD_STEP, CMD_STEP_AT, _CommandWire

    w = _CommandWire(max_requests=4, max_seq_len=16, device=torch.device("cpu"))
    sent = []
    w.broadcast = lambda t: sent.append(t.clone())
    w.send(CMD_STEP, 3, (7, 9), torch.tensor([[1], [2]]))
    w.send(CMD_STEP, 4, (7, 9), torch.tensor([[3], [4]]))
    w.send(CMD_STEP_AT, 0, (7, 9), torch.tensor([[5], [6]]), positions=(5, 6))
    w.send(CMD_STEP, 6, (7, 8), torch.tensor([[5], [6]]))
    w.send(CMD_RELEASE, 0, (7, 8))
    frames = iter(sent)
    r = _CommandWire(max_requests=4, max_seq_len=16, device=torch.device("cpu"))
    r.broadcast = lambda t: t.copy_(next(frames))
    a, b, c, d, e = (r.receive() for _ in range(5))
    assert a.ids == b.ids == c.ids == (7, 9) and a.ids is b.ids and b.ids is c.ids
    assert c.positions == (5, 6) and c.tokens.tolist() == [[5], [6]]
    assert d.ids == (7, 8) and d.ids is not a.ids and e.ids is d.ids
    assert all(type(v) is int for v in d.ids)


def test_cache_validate_at_agrees_with_per_request_validate():
    """validate_at(ids, positions, n) raises exactly when validate((r,), p, n)
    raises for some request, and also for duplicate ids."""
    import random

    rng = random.Random(5)
    for trial in range(300):
        c = cache(layer_ids=(2, 4, 6), max_requests=6, max_seq_len=12)
        ids = tuple(rng.sample(range(20), 4))
        c.reserve(ids)
        level = {}
        for r in ids:  # each request at its own length; some with a layer ahead
            level[r] = n = rng.randrange(0, 8)
            if n:
                c.advance((r,), n)
            if rng.random() < 0.15:
                c.append(rng.choice((2, 4, 6)), (r,), kv(1, 1), kv(1, 1), n)
        if rng.random() < 0.9:  # mostly distinct reserved ids
            q = tuple(rng.sample(ids, rng.randrange(1, 5)))
        else:
            q = tuple(rng.choice(ids + (99,)) for _ in range(rng.randrange(1, 5)))
        # mostly each request's own position
        pos = tuple(level.get(r, 0) if rng.random() < 0.9 else rng.randrange(-1, 12) for r in q)
        count = rng.choice((1, 1, 1, 2, 0))

        def per_request():
            for r, p in zip(q, pos):
                c.validate((r,), p, count)

        want = None
        try:
            per_request()
        except CacheError as e:
            want = e
        dup = len(set(q)) != len(q)
        if want is None and not dup:
            c.validate_at(q, pos, count)
        else:
            with pytest.raises(CacheError):
                c.validate_at(q, pos, count)
    with pytest.raises(CacheError, match="one position per request"):
        c.validate_at(ids[:2], (0,), 1)
