"""Progressive P/D protocol pieces on CPU: state machine, schedules, stages, paced wire."""
import pytest
import torch

from sparsecache_b200.serving.progressive import (
    Document,
    ProgressivePDPhase,
    ProgressivePDRequestState,
    TrancheStager,
    accepted_prefix_length,
    lexical_scores,
    ranked_document_indices,
    stage_document_sets,
    van_der_corput_order,
)


def test_state_machine_protocol():
    s = ProgressivePDRequestState(priority_pages=(3, 1, 2, 0), anchor_pages=1, max_draft_tokens=2)
    with pytest.raises(RuntimeError):
        s.record_draft_token(7)  # before the anchor
    s.record_page_completion({1})  # out of order: no visible prefix yet
    assert s.phase == ProgressivePDPhase.WAIT_ANCHOR and s.visible_priority_pages == ()
    s.record_page_completion({3})
    assert s.phase == ProgressivePDPhase.DRAFT_WHILE_LOADING
    assert s.visible_priority_pages == (3, 1) and s.visible_fraction == 0.5
    with pytest.raises(ValueError):
        s.record_page_completion({3})  # duplicate
    with pytest.raises(ValueError):
        s.record_page_completion({9})  # unknown
    s.record_draft_token(11)
    s.record_draft_token(12)
    with pytest.raises(RuntimeError):
        s.record_draft_token(13)  # limit
    with pytest.raises(RuntimeError):
        s.record_final_verification(1, 5)  # not all KV yet
    s.record_page_completion({0, 2})
    assert s.phase == ProgressivePDPhase.READY_TO_VERIFY
    with pytest.raises(RuntimeError):
        s.record_page_completion(set())
    s.record_final_verification(1, 99)
    assert s.external_token_ids == [11, 99] and s.verifier_calls == 1
    with pytest.raises(RuntimeError):
        s.record_final_verification(0, 1)  # the verifier runs once
    s.finish()
    assert s.phase == ProgressivePDPhase.FINISHED
    with pytest.raises(ValueError):
        ProgressivePDRequestState(priority_pages=(1, 1), anchor_pages=1, max_draft_tokens=1)


def _docs():
    texts = ["cats and dogs", "the paris tower", "dogs bark loud", "paris france capital", "random words"]
    docs, cursor = [], 4
    for i, t in enumerate(texts):
        n = 10 + 5 * i
        docs.append(Document(tuple(range(n)), t, supporting=(i in (1, 3)), start=cursor, end=cursor + n))
        cursor += n
    return docs


def test_schedules_and_stages():
    docs = _docs()
    scores = lexical_scores("capital of paris", docs)
    assert scores[3] > scores[1] > 0 and scores[0] == 0
    assert ranked_document_indices("query", question="capital of paris", documents=docs, random_seed=0)[:2] == [3, 1]
    assert ranked_document_indices("sequential", question="", documents=docs, random_seed=0) == [0, 1, 2, 3, 4]
    assert van_der_corput_order(8) == [0, 4, 2, 6, 1, 5, 3, 7]
    assert ranked_document_indices("oracle", question="", documents=docs, random_seed=0)[:2] == [1, 3]
    assert ranked_document_indices("support_last", question="", documents=docs, random_seed=0)[-2:] == [1, 3]
    r1 = ranked_document_indices("random", question="", documents=docs, random_seed=5)
    assert sorted(r1) == list(range(5)) and r1 == ranked_document_indices("random", question="", documents=docs,
                                                                           random_seed=5)
    pa = ranked_document_indices("p_attention", question="", documents=docs, random_seed=0,
                                 attention_scores=[0.1, 0.5, 0.2, 0.9, 0.0])
    assert pa[0] == 3
    with pytest.raises(ValueError):
        ranked_document_indices("p_attention", question="", documents=docs, random_seed=0)
    ranking = [3, 1, 0, 2, 4]
    stages = stage_document_sets(ranking, docs, (0.1, 0.4, 1.0))
    total = sum(len(d.token_ids) for d in docs)
    assert stages[0] == {3} and sum(len(docs[i].token_ids) for i in stages[1]) >= 0.4 * total
    assert stages[-1] == set(range(5))
    assert accepted_prefix_length([1, 2, 3], [1, 2, 4]) == 2 and accepted_prefix_length([], [1]) == 0


def test_stager_layout_and_paced_wire():
    docs = _docs()
    T = 4 + sum(len(d.token_ids) for d in docs) + 3
    source = torch.zeros(2, 2, 1, T, 4)
    ranking = [3, 1, 0, 2, 4]
    stages = stage_document_sets(ranking, docs, (0.1, 0.5, 1.0))
    now = [100.0]
    slept = []

    def clock():
        return now[0]

    def sleep(dt):
        slept.append(dt)
        now[0] += dt

    class Slot:
        data = torch.zeros(2, 2, 1, T, 4)

    st = TrancheStager(source, Slot(), prefix_tokens=4, documents=docs, suffix_tokens=3, ranking=ranking,
                       selected_sets=stages, transport_gbps=1.0, clock=clock, sleep=sleep)
    # stage 0 = prefix + suffix + first ranked doc; destinations are contiguous
    assert st.stages[0].ranges[0] == (0, 4) and st.stages[0].ranges[1] == (T - 3, T)
    assert st.stages[0].ranges[2] == (docs[3].start, docs[3].end)
    assert st.stages[-1].destination_end == T
    assert sorted(st.compact_positions) == list(range(T))
    st.launch(0)
    wire_s = st.stage_bytes(0) * 8 / 1e9
    assert abs(st.wire_ready_at[0] - (100.0 + wire_s)) < 1e-12
    st.poll_ready_copies()
    assert not st.physical_launched[0]
    now[0] += wire_s
    st.poll_ready_copies()
    assert st.physical_launched[0] and st.stage_copy_ready(0)
    # eager serial wire: cumulative deadlines on one wire
    st2 = TrancheStager(source, Slot(), prefix_tokens=4, documents=docs, suffix_tokens=3, ranking=ranking,
                        selected_sets=stages, transport_gbps=1.0, eager_serial_wire=True, clock=clock, sleep=sleep)
    st2.launch(0)
    assert all(st2.launched)
    ends = st2.wire_ready_at
    assert ends[0] < ends[1] < ends[2]
    assert abs((ends[2] - ends[1]) - st2.stage_bytes(2) * 8 / 1e9) < 1e-9
    with pytest.raises(RuntimeError):
        TrancheStager(source, Slot(), prefix_tokens=4, documents=docs, suffix_tokens=3, ranking=ranking,
                      selected_sets=stages, transport_gbps=1.0, eager_serial_wire=True,
                      clock=clock, sleep=sleep).launch(1)


def test_whole_cache_encoders_and_visibility_masks():
    """Independent encoding equals each segment prefilled alone at its target offset (RoPE attention
    depends on relative positions only); masks open the prefix, the chosen documents and the suffix."""
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.serving.progressive import (Document, encode_contiguous_cache, encode_independent_cache,
                                                      pd_visibility_mask, prefix_visibility_mask, visible_slot_map)

    model = LlamaOracle.random_init(get_model_config("tiny"), seed=2, std=0.05)
    g = torch.Generator().manual_seed(0)
    prefix = torch.randint(4, 1024, (5,), generator=g).tolist()
    docs, start = [], len(prefix)
    for n in (7, 4, 9):
        ids = tuple(torch.randint(4, 1024, (n,), generator=g).tolist())
        docs.append(Document(ids, start=start, end=start + n))
        start += n
    cache = encode_independent_cache(model, prefix, docs)
    assert cache[1][0].shape == (1, 2, start, 64)
    d = docs[2]
    _, alone = model.prefill(list(d.token_ids), start=d.start)
    for layer in range(2):
        assert torch.allclose(cache[layer][0][:, :, d.start:d.end], alone[layer][0], atol=1e-4, rtol=1e-4)
        assert torch.allclose(cache[layer][1][:, :, d.start:d.end], alone[layer][1], atol=1e-4, rtol=1e-4)
    full = encode_contiguous_cache(model, prefix + [t for x in docs for t in x.token_ids])
    assert torch.allclose(full[0][0][:, :, :5], cache[0][0][:, :, :5], atol=1e-5)  # the prefix is the same prefill
    m = prefix_visibility_mask(len(prefix), docs, {1})
    assert m.shape == (1, start) and m[0, :5].all() and m[0, docs[1].start:docs[1].end].all()
    assert int(m.sum()) == 5 + 4
    pm = pd_visibility_mask(len(prefix), docs, 3, {0, 2})
    assert pm.shape == (1, start + 3) and pm[0, -3:].all() and int(pm.sum()) == 5 + 7 + 9 + 3
    sm = visible_slot_map(m)
    assert sm.dtype == torch.int32 and sm.tolist() == list(range(5)) + list(range(docs[1].start, docs[1].end))


def test_native_tranche_packing_matches_concatenation():
    """Each stage's pinned block holds its token ranges back to back, as a concatenation along tokens."""
    from sparsecache_b200 import ops
    from sparsecache_b200.serving.progressive import Document, TrancheStager

    g = torch.Generator().manual_seed(0)
    src = torch.randn(3, 2, 2, 100, 8, generator=g).to(torch.bfloat16)
    docs, at = [], 4
    for n in (20, 30, 36):
        docs.append(Document(tuple(range(n)), start=at, end=at + n))
        at += n
    st = TrancheStager(src, None, prefix_tokens=4, documents=docs, suffix_tokens=10, ranking=[2, 0, 1],
                       selected_sets=[{2}, {2, 0}, {0, 1, 2}])
    st.pack(n_threads=3)
    for stage, block in zip(st.stages, st._packed):
        want = torch.cat([src[:, :, :, b:e] for b, e in stage.ranges], dim=3)
        assert torch.equal(block, want)
    ext = ops.ext()
    rows = src.view(-1, 100, 8)
    out = torch.empty(rows.shape[0], 5, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ext.pack_token_ranges(rows, [98], [103], out, 2)  # range past the tokens
    with pytest.raises(RuntimeError):
        ext.pack_token_ranges(rows, [0], [4], out, 2)  # width differs from the destination
