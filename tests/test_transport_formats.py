"""Payload identity formats, revealed-only packing state, verifiers and the
guarded peer adapter (CPU; reference tests test_r3_reference_a2av.py,
test_r4_reference_full_moe.py and test_r6_mscclpp_adapter.py re-expressed)."""

from types import SimpleNamespace

import numpy as np
import pytest

from revealaiccl_b200.transport.formats import (
    ProgressivePackingState, RouterAssignment, build_destination_layout, identity_checksum,
    identity_checksum_vec, pack_destination_layout, pack_forward_payload, pack_return_payload, payload_checksum,
    row_digest, verify_forward_payload, verify_received_records, verify_return_and_combine)
from revealaiccl_b200.transport.peer_adapter import (COUNT_HEADER_BYTES, HostPeerMemory, PeerCommittedAdapter,
                                                     RegisteredBufferLayout)

PASS = SimpleNamespace(accepted=True, applied_actions=1)
FAIL = SimpleNamespace(accepted=False, applied_actions=0)


def _assign(token, dst, expert, chunk=0, off=0, src=0):
    return RouterAssignment(token, src, dst, expert, chunk, off, token * 3)


def test_checksum_linear_and_vectorised():
    rows = np.array([[5, 1, 0, 3, 2, 7, 9, 11], [2 ** 62, 0, 1, 1, 0, 0, 0, 5]], dtype=np.int64)
    vec = identity_checksum_vec(rows)
    assert [identity_checksum(r) for r in rows.tolist()] == vec.tolist()
    base = identity_checksum((5, 1, 0, 0, 2, 7, 9, 11))
    assert (base + 0 * 1_000_037 + 3 * 1_000_081) % ((1 << 63) - 25) == vec[0]


def test_row_digest_is_order_dependent_and_detects_bit_flip():
    x = np.arange(64, dtype=np.float32).reshape(2, 32)
    d = row_digest(x)
    assert d[0] != d[1]
    y = x.copy()
    y[0, [3, 4]] = y[0, [4, 3]]
    assert row_digest(y)[0] != d[0]
    z = x.copy()
    z.view(np.uint32)[1, 7] ^= 1
    assert row_digest(z)[1] != d[1]


def test_layout_counts_offsets_and_sort():
    a = [_assign(30, 1, 1), _assign(10, 0, 0), _assign(20, 1, 3), _assign(11, 0, 2)]
    lay = build_destination_layout(a, world_size=2, source_rank=0, chunk_ids=(0,))
    assert lay.sendcounts_tokens == (2, 2) and lay.offsets_tokens == (0, 2)
    assert [x.token_id for x in lay.destination_lists[0]] == [10, 11]
    packed = pack_destination_layout(lay)
    assert packed.records.shape == (4, 8) and not packed.records.flags.writeable
    assert all(payload_checksum(r[:7]) == r[7] for r in packed.records.tolist())


@pytest.mark.parametrize("bad,msg", [
    (_assign(1, 0, 0, src=1), "source"), (_assign(1, 0, 0, chunk=3), "unrevealed"),
    (_assign(1, 5, 5), "outside"), (_assign(1, 1, 2), "expert-derived")])
def test_layout_fails_closed(bad, msg):
    with pytest.raises(ValueError, match=msg):
        build_destination_layout([bad], world_size=2, source_rank=0, chunk_ids=(0,))


def test_layout_zero_sized_pair_and_empty_shard():
    lay = build_destination_layout([_assign(1, 0, 0), _assign(2, 0, 2)], world_size=2, source_rank=0, chunk_ids=(0,))
    assert lay.sendcounts_tokens == (2, 0)
    empty = build_destination_layout([], world_size=2, source_rank=0, chunk_ids=(0,))
    assert empty.sendcounts_tokens == (0, 0) and pack_destination_layout(empty).records.shape == (0, 8)


def test_packing_state_counters():
    st = ProgressivePackingState(world_size=2, source_rank=0, max_chunks=4)
    st.mark_completed(0, [_assign(1, 0, 0, chunk=0)])
    with pytest.raises(ValueError, match="future"):
        st.build_delta_layout((1,))
    assert st.future_access_attempts == 1
    with pytest.raises(ValueError, match="unrevealed"):
        st.build_delta_layout((0,))
    assert st.unrevealed_execution == 1
    st.reveal(0)
    st.build_delta_layout((0,))
    with pytest.raises(ValueError, match="stale"):
        st.build_delta_layout((0,))
    assert st.stale_dispatch == 1
    st.mark_completed(1, [_assign(1, 0, 0, chunk=1)])
    st.reveal(1)
    with pytest.raises(ValueError, match="duplicate"):
        st.build_delta_layout((1,))
    assert st.duplicate_dispatch == 1
    with pytest.raises(ValueError, match="incomplete"):
        st.reveal(2)


def test_receive_verifier_detects_loss_corruption_wrong_destination():
    recs = pack_destination_layout(build_destination_layout(
        [_assign(1, 0, 0), _assign(2, 0, 2)], world_size=2, source_rank=0, chunk_ids=(0,))).records
    expected = {int(r[0]): tuple(int(x) for x in r) for r in recs}
    assert verify_received_records(recs, destination_rank=0, expected_by_token=expected)["pass"]
    bad = recs.copy()
    bad[0, 6] += 1
    res = verify_received_records(bad, destination_rank=0, expected_by_token=expected)
    assert not res["pass"] and res["corruption"] >= 1
    res = verify_received_records(recs[:1], destination_rank=0, expected_by_token=expected)
    assert res["lost"] == 1
    res = verify_received_records(recs, destination_rank=1, expected_by_token=expected)
    assert res["wrong_destination"] == 2


def test_forward_return_roundtrip_and_corruption():
    lay = build_destination_layout([_assign(10, 0, 0), _assign(11, 1, 1, off=1)], world_size=2,
                                   source_rank=0, chunk_ids=(0,))
    feats = {10: np.array([1.0, 2.0], np.float32), 11: np.array([3.0, 4.0], np.float32)}
    pay = pack_forward_payload(lay, features_by_token=feats, original_position_by_token={10: 0, 11: 1})
    assert pay.sendcounts_tokens == (1, 1)
    assert verify_forward_payload(pay.metadata[:1], pay.features[:1], destination_rank=0, world_size=2)["pass"]
    bad = pay.features[:1].copy()
    bad[0, 0] += 1
    assert not verify_forward_payload(pay.metadata[:1], bad, destination_rank=0, world_size=2)["pass"]
    outs = np.array([[5.0, 6.0]], np.float32)
    ret = pack_return_payload(pay.metadata[:1], outs, expert_rank=0, world_size=2)
    comb, res = verify_return_and_combine(ret.metadata, ret.outputs, origin_rank=0, recvcounts_tokens=(1, 0),
                                          expected_expert_by_token={10: 0}, expected_position_by_token={10: 0},
                                          expected_output_by_token={10: outs[0]}, total_tokens=1)
    assert res["pass"] and np.array_equal(comb, outs)
    meta = ret.metadata.copy()
    meta[0, 7] += 1
    _, res = verify_return_and_combine(meta, ret.outputs, origin_rank=0, recvcounts_tokens=(1, 0),
                                       expected_expert_by_token={10: 0}, expected_position_by_token={10: 0},
                                       expected_output_by_token={10: outs[0]}, total_tokens=1)
    assert not res["pass"] and res["corruption"] == 1


def _packed(dst_counts, src=0, chunks=(0,)):
    a = []
    tok = 100
    for dst, n in enumerate(dst_counts):
        for _ in range(n):
            a.append(_assign(tok, dst, dst, src=src))
            tok += 1
    return pack_destination_layout(build_destination_layout(a, world_size=len(dst_counts), source_rank=src,
                                                            chunk_ids=chunks))


def test_adapter_offsets_header_only_and_fail_closed():
    lay = RegisteredBufferLayout(world_size=4, max_descriptors=3, max_tokens_per_peer_descriptor=8)
    ad = PeerCommittedAdapter(rank=1, layout=lay)
    acts = ad.commit_descriptor(_packed([2, 0, 0, 1], src=1), descriptor_id=0, guard_decision=PASS,
                                completed_chunks=(0,), revealed_chunks=(0,))
    # empty local slot skipped, empty remote (rank 2) is header-only
    assert [a.dst_rank for a in acts] == [0, 2, 3]
    assert acts[1].token_count == 0 and acts[1].physical_bytes == COUNT_HEADER_BYTES
    assert acts[0].dst_offset == lay.receive_offset(0, 1)
    with pytest.raises(ValueError, match="stale"):
        ad.commit_descriptor(_packed([1, 0, 0, 0], src=1), descriptor_id=0, guard_decision=PASS,
                             completed_chunks=(0,), revealed_chunks=(0,))
    with pytest.raises(ValueError, match="PASS"):
        ad.commit_descriptor(_packed([1, 0, 0, 0], src=1), descriptor_id=1, guard_decision=FAIL,
                             completed_chunks=(0,), revealed_chunks=(0,))
    with pytest.raises(ValueError, match="future"):
        ad.commit_descriptor(_packed([1, 0, 0, 0], src=1), descriptor_id=1, guard_decision=PASS,
                             completed_chunks=(), revealed_chunks=())
    with pytest.raises(ValueError, match="unrevealed"):
        ad.commit_descriptor(_packed([1, 0, 0, 0], src=1), descriptor_id=1, guard_decision=PASS,
                             completed_chunks=(0,), revealed_chunks=())
    c = ad.counters()
    assert c["stale_action"] == 1 and c["future_access"] == 1 and c["unrevealed_access"] == 1
    with pytest.raises(ValueError, match="capacity"):
        ad.commit_descriptor(_packed([9, 0, 0, 0], src=1), descriptor_id=2, guard_decision=PASS,
                             completed_chunks=(0,), revealed_chunks=(0,))


def test_host_peer_memory_put_signal_receive():
    lay = RegisteredBufferLayout(world_size=2, max_descriptors=2, max_tokens_per_peer_descriptor=4)
    mem = HostPeerMemory(lay)
    packed = _packed([1, 2])
    ad = PeerCommittedAdapter(rank=0, layout=lay)
    acts = ad.commit_descriptor(packed, descriptor_id=0, guard_decision=PASS, completed_chunks=(0,),
                                revealed_chunks=(0,))
    for a in acts:
        mem.stage(0, a, packed, packed.offsets_tokens[a.dst_rank])
        mem.put_and_signal(a)
    assert mem.wait(1, 0, 0)
    got = mem.receive(1, 0, 0)
    assert np.array_equal(got, packed.records[1:3])
    assert mem.counters["put_calls"] == 2 and mem.counters["bytes_transferred"] == 16 + 3 * 64
