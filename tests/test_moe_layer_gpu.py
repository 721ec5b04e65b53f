"""GPU tests of the progressive MoE data plane on one B200 (world size 1).

Every kernel result is compared against a plain PyTorch fp32 reference of the
same op; the full layer is checked by the fail-closed checker (identity rows,
return rows, expert outputs, combined output, packing counters and the
differential replay of the device control plane), and the early and delayed
arms must produce bit-identical outputs.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _small(dtype="fp32", act="relu", k=2, **kw):
    from revealaiccl_b200.moe.config import MoELayerConfig

    return MoELayerConfig(
        name=f"small_{dtype}_{act}", tokens_per_rank=1024, hidden=256, experts=4, top_k=k,
        chunk_sizes=(128,) * 8, ffn_hidden=256 if act != "swiglu" else 128, out_dim=256,
        activation=act, dtype=dtype, placement="contiguous",
        gate_mode="topk_softmax" if k > 1 else "none", router_init="unit_logits",
        expert_init="normal002", **kw)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("E,k", [(4, 1), (8, 2), (64, 6)])
def test_router_kernel_matches_fp32_oracle(dtype, E, k):
    from revealaiccl_b200.ops._native import kernels

    torch.manual_seed(0)
    dev = torch.device("cuda")
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    T, D = 700, 512
    x = torch.randn(T, D, device=dev).to(dt)
    w = (torch.randn(E, D, device=dev) / D ** 0.5).to(dt)
    b = torch.randn(E, device=dev) * 0.1
    ids = torch.zeros(T, k, dtype=torch.int32, device=dev)
    gates = torch.zeros(T, k, device=dev)
    kernels().router_topk(x, w, b, None, None, 0, T, k, 1, 1, ids, gates)
    logits = x.float() @ w.float().t() + b
    pos = torch.arange(T, device=dev)
    logits[pos, pos % E] = float("-inf")
    vals, ref = torch.sort(logits, dim=-1, descending=True, stable=True)
    ref = ref[:, :k].int()
    gap_ok = (vals[:, :k] - logits.gather(1, ids.long())).abs() <= 1e-4 * (1 + vals[:, :1].abs())
    assert ((ref == ids).all(dim=1) | gap_ok.all(dim=1)).all()
    ref_g = torch.softmax(vals[:, :k], dim=-1)
    same = (ref == ids).all(dim=1)
    torch.testing.assert_close(gates[same], ref_g[same], atol=1e-4, rtol=1e-4)


def test_router_ties_pick_smaller_expert():
    from revealaiccl_b200.ops._native import kernels

    dev = torch.device("cuda")
    T, D, E = 64, 64, 8
    x = torch.zeros(T, D, device=dev)
    w = torch.zeros(E, D, device=dev)
    b = torch.zeros(E, device=dev)
    b[3] = b[5] = 1.0
    ids = torch.zeros(T, 2, dtype=torch.int32, device=dev)
    gates = torch.zeros(T, 2, device=dev)
    kernels().router_topk(x, w, b, None, None, 0, T, 2, 0, 0, ids, gates)
    assert (ids[:, 0] == 3).all() and (ids[:, 1] == 5).all()


def test_feature_digest_matches_numpy():
    from revealaiccl_b200.ops._native import kernels
    from revealaiccl_b200.transport.formats import row_digest

    dev = torch.device("cuda")
    x = torch.randn(257, 384, device=dev)
    dig = torch.empty(257, dtype=torch.int64, device=dev)
    kernels().feature_digest(x, dig)
    assert np.array_equal(dig.cpu().numpy(), row_digest(x.cpu().numpy()))


@pytest.mark.parametrize("dtype,act,k", [("fp32", "relu", 1), ("fp32", "gelu", 2), ("bf16", "swiglu", 2)])
def test_layer_world1_early_delayed_identical_and_verified(dtype, act, k):
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(_small(dtype, act, k), timeout_s=5.0)
    try:
        layer.forward("early")
        rep_e = layer.verify()
        out_e = layer.out.clone()
        layer.forward("delayed")
        rep_d = layer.verify()
        assert rep_e["pass"] and rep_d["pass"]
        assert torch.equal(out_e, layer.out)
        assert rep_e["control"]["total"] == layer.cfg.n_desc
    finally:
        layer.close()


def test_r4_reference_config_world1():
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(preset("r4_reference"), timeout_s=5.0)
    try:
        layer.forward("early")
        rep = layer.verify()
        assert rep["pass"], rep["violations"]
        assert rep["forward"]["tokens"] == 4096
        out_e = layer.out.clone()
        layer.forward("delayed")
        assert layer.verify()["pass"]
        assert torch.equal(out_e, layer.out)
    finally:
        layer.close()


def test_r4_case_families_world1():
    from revealaiccl_b200.moe.config import CASE_ORDER, r4_case
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    for case in CASE_ORDER:
        layer = ProgressiveMoELayer(r4_case(case), timeout_s=5.0)
        try:
            layer.forward("early")
            rep = layer.verify()
            assert rep["pass"], (case, rep["violations"])
        finally:
            layer.close()


def test_graph_capture_replay_repeated_calls():
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(_small("bf16", "swiglu", 2), timeout_s=5.0)
    try:
        layer.forward("early")
        ref = layer.out.clone()
        n = layer.capture("early")
        assert n >= 7  # reset, front end (or its step kernels), plan + tile tables, return meta, 2 GEMMs, combine
        for _ in range(3):
            layer.replay()
        torch.cuda.synchronize()
        rep = layer.verify()
        assert rep["pass"] and rep["epoch"] == 4
        assert torch.equal(ref, layer.out)
    finally:
        layer.close()


@pytest.mark.parametrize("case", ["balanced", "skewed", "empty_shard", "multiple_progressive_shards"])
def test_warp_control_plane_matches_cta_kernel(case):
    """The single-warp control kernel and the CTA kernel make the same decisions,
    leave the same scheduler state and write the same log rows."""
    from revealaiccl_b200.moe.config import r4_case
    from revealaiccl_b200.moe.layer import LOG_HEADER, ProgressiveMoELayer

    res = {}
    for path in ("auto", "serial"):
        layer = ProgressiveMoELayer(r4_case(case), timeout_s=5.0, control_path=path, frontend="steps")
        try:
            layer.forward("early")
            rep = layer.verify()
            assert rep["pass"], (path, rep["violations"])
            lay = layer.control_layout
            blob = layer.tensors["ctl_blob"].cpu()
            log = layer.tensors["ctl_log"].cpu().view(layer.cfg.n_desc, layer.log_stride)
            res[path] = (blob[int(lay["state_begin"]):int(lay["state_end"])].clone(),
                         torch.cat([log[:, :8], log[:, LOG_HEADER:]], dim=1).clone(),
                         int(log[0, 15]), layer.out.clone())
        finally:
            layer.close()
    assert res["auto"][2] == 1 and res["serial"][2] == 0  # which kernel ran
    assert torch.equal(res["auto"][0], res["serial"][0])
    assert torch.equal(res["auto"][1], res["serial"][1])
    assert torch.equal(res["auto"][3], res["serial"][3])


@pytest.mark.parametrize("name", ["r4_reference", "full_tf32", "r4:skewed", "r4:empty_shard",
                                  "r4:multiple_progressive_shards"])
def test_persistent_frontend_matches_step_pipeline(name):
    """The persistent cooperative front end (packed control path) and the
    one-launch-per-step pipeline (byte-per-entry control path) produce identical
    outputs, control state and log rows, in both arms."""
    from revealaiccl_b200.moe.config import preset, r4_case
    from revealaiccl_b200.moe.layer import LOG_HEADER, ProgressiveMoELayer

    cfg = r4_case(name[3:]) if name.startswith("r4:") else preset(name)
    res = {}
    for fe in ("persistent", "steps"):
        layer = ProgressiveMoELayer(cfg, timeout_s=5.0, frontend=fe)
        try:
            outs = []
            for arm in ("early", "delayed"):
                layer.forward(arm)
                rep = layer.verify()
                assert rep["pass"], (fe, arm, rep["violations"])
                outs.append(layer.out.clone())
            assert layer.runner.persistent_frontend() == (fe == "persistent")
            if fe == "persistent":
                log15 = layer.tensors["ctl_log"].cpu().view(layer.cfg.n_desc, layer.log_stride)[:, 15]
                assert bool((log15 == 2).all())  # every trigger ran on the packed path
            lay = layer.control_layout
            blob = layer.tensors["ctl_blob"].cpu()
            log = layer.tensors["ctl_log"].cpu().view(layer.cfg.n_desc, layer.log_stride)
            res[fe] = (outs, blob[int(lay["state_begin"]):int(lay["state_end"])].clone(),
                       torch.cat([log[:, :8], log[:, LOG_HEADER:]], dim=1).clone())
        finally:
            layer.close()
    for i in range(2):
        assert torch.equal(res["persistent"][0][i], res["steps"][0][i])
    assert torch.equal(res["persistent"][0][0], res["persistent"][0][1])
    assert torch.equal(res["persistent"][1], res["steps"][1])
    assert torch.equal(res["persistent"][2], res["steps"][2])


def test_cta_pair_gemms_leave_layer_output_unchanged():
    """The layer's GEMMs on the CTA-pair kernel give bit-identical outputs."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    outs = []
    for pair in (True, False):
        layer = ProgressiveMoELayer(preset("full_tf32").with_overrides(tokens_per_rank=2048, chunk_sizes=(256,) * 8),
                                    timeout_s=5.0, gemm_pair=pair)
        try:
            layer.forward("early")
            assert layer.verify()["pass"]
            outs.append(layer.out.clone())
        finally:
            layer.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.gpu
def test_programmatic_dependent_launch_matches_plain_launches():
    """Plan, GEMMs and combine launched as programmatic dependents give the same
    output as ordinary stream-ordered launches, over repeated calls and graph
    replay (the return-signal handoff counters stay in step)."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    outs = {}
    for pdl in (True, False):
        layer = ProgressiveMoELayer(preset("full_tf32").with_overrides(tokens_per_rank=2048, chunk_sizes=(256,) * 8),
                                    timeout_s=5.0, pdl=pdl)
        try:
            for arm in ("early", "delayed", "early"):
                layer.forward(arm)
                assert layer.verify()["pass"], (pdl, arm)
            layer.capture("early")
            for _ in range(3):
                layer.replay()
            assert layer.verify()["pass"]
            sync = layer.tensors["ret_sync"].cpu().tolist()
            calls = int(layer.tensors["epoch"].cpu().item())
            assert sync[0] == calls and sync[1] == 2 * calls  # one election and two parts per call
            outs[pdl] = layer.out.clone()
        finally:
            layer.close()
    assert torch.equal(outs[True], outs[False])


@pytest.mark.gpu
def test_streamed_inputs_match_resident_calls():
    """The end-to-end call streams the token batch chunk by chunk into the running
    front end (the workers digest the rows they route); outputs, verification and
    digests equal the resident path's, eagerly and through the captured graph."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(preset("full_tf32").with_overrides(tokens_per_rank=2048, chunk_sizes=(256,) * 8),
                                timeout_s=5.0)
    try:
        layer.forward("early")
        torch.cuda.synchronize()
        assert layer.runner.persistent_frontend()
        ref_out = layer.out.clone()
        ref_digest = layer.feat_digest.clone()
        host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
        host_in.copy_(layer.inputs.tokens.cpu())
        host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        for i in range(3):
            layer.inputs.tokens.zero_()  # the call must bring its own rows
            layer(host_in, host_out, arm="early")
            torch.cuda.synchronize()
            rep = layer.verify()
            assert rep["pass"], (i, rep["violations"])
            assert torch.equal(host_out, ref_out.cpu())
            assert torch.equal(layer.feat_digest, ref_digest)
        layer.capture("early")
        layer.inputs.tokens.zero_()
        layer(host_in, host_out, arm="early")  # graph replay with streamed inputs
        torch.cuda.synchronize()
        assert layer.verify()["pass"] and torch.equal(host_out, ref_out.cpu())
        layer.forward("delayed")  # a resident call after streamed ones
        assert layer.verify()["pass"]
        assert layer.runner.calls() == int(layer.tensors["epoch"].item())
    finally:
        layer.close()


@pytest.mark.gpu
def test_streamed_copies_start_inside_the_callers_window():
    """A timed end-to-end region opened on the comm stream must contain the
    call's host-to-device copies: the copy stream waits for everything already
    enqueued on the comm stream.  A 5 ms device sleep sits on the comm stream
    before the start event; copies that did not wait for it would finish
    before the start event."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(preset("full_tf32").with_overrides(tokens_per_rank=2048, chunk_sizes=(256,) * 8),
                                timeout_s=5.0)
    try:
        layer.forward("early")
        torch.cuda.synchronize()
        host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
        host_in.copy_(layer.inputs.tokens.cpu())
        host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        cs = layer.comm_stream
        for graph in (False, True):
            if graph:
                layer.capture("early")
            s = torch.cuda.Event(enable_timing=True)
            copied = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(cs):
                torch.cuda._sleep(int(5e-3 * 1.9e9))  # ~5 ms at the maximum SM clock
            s.record(cs)
            layer(host_in, host_out, arm="early")
            copied.record(layer.copy_stream)  # after the call's last chunk copy
            torch.cuda.synchronize()
            assert s.elapsed_time(copied) > 0.0, graph
            assert layer.verify()["pass"]
    finally:
        layer.close()


# The bf16 benchmark shapes with their full expert widths, expert counts,
# top-k, chunk counts and gate modes, on fewer tokens per rank.
BASELINE_SHAPES = {
    "skewed_bf16": dict(tokens_per_rank=2048, chunk_sizes=(128,) * 16),
    "mixtral_8x7b": dict(tokens_per_rank=2048, chunk_sizes=(64,) * 32),
    "deepseek_v2_lite": dict(tokens_per_rank=2048, chunk_sizes=(128,) * 16),
}


@pytest.mark.parametrize("name", sorted(BASELINE_SHAPES))
def test_baseline_shapes_world1_verified(name):
    """SwiGLU experts at the benchmark widths (Mixtral 4096->14336->4096,
    DeepSeek-V2-Lite 64 experts top-6 2048->1408->2048, skewed 16 experts with
    Zipf bias and a hot phase) pass the fail-closed checker against the fp32
    oracle, and the early and delayed arms give identical outputs."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    cfg = preset(name, **BASELINE_SHAPES[name])
    layer = ProgressiveMoELayer(cfg, timeout_s=10.0)
    try:
        layer.forward("early")
        rep = layer.verify()
        assert rep["pass"], rep["violations"]
        assert rep["forward"]["tokens"] == cfg.tokens_per_rank * cfg.top_k
        out_e = layer.out.clone()
        layer.forward("delayed")
        assert layer.verify()["pass"]
        assert torch.equal(out_e, layer.out)
    finally:
        layer.close()


def _revealed_prefix(layer, c):
    """Everything the layer produced for router chunks 0..c and descriptors
    0..c: expert ids and gates of those rows, the control-log decision rows
    (without their phase clocks) and the forward identity rows and features
    each (local expert, source) region received from those descriptors."""
    cfg = layer.cfg
    off = cfg.chunk_offsets
    T, W, S = cfg.tokens_per_rank, layer.world, layer.slots
    torch.cuda.synchronize()
    log = layer.tensors["ctl_log"].view(cfg.n_desc, layer.log_stride).cpu()
    counts = layer._region("recv_count", (S, W, cfg.n_desc), torch.int32).cpu()
    meta = layer._region("recv_meta", (S, W, T, 9), torch.int64).cpu()
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    feat = layer._region("recv_feat", (S, W, T, cfg.hidden), dt).cpu()
    rows = []
    for s in range(S):
        for src in range(W):
            n = int(counts[s, src, :c + 1].sum())
            rows.append((meta[s, src, :n].clone(), feat[s, src, :n].clone()))
    return {
        "ids": layer.expert_ids[:off[c + 1]].cpu(), "gates": layer.gates[:off[c + 1]].cpu(),
        "log": torch.cat([log[:c + 1, :8], log[:c + 1, 16:]], dim=1),
        "rows": rows,
    }


def test_hidden_future_perturbation_leaves_revealed_prefix_unchanged():
    """Revealed-only on the device path: changing the token rows and the
    router logit bias of every chunk after chunk c between two calls must not
    change anything the layer decided or sent for chunks (descriptors) 0..c:
    routing, control-plane decisions and dispatched identity rows are equal,
    while the later chunks' routing does change."""
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    c = 2
    layer = ProgressiveMoELayer(_small("fp32", "gelu", 2, case_bias=(0.0, 0.0, 0.0, 0.0)), timeout_s=5.0)
    try:
        assert c < layer.cfg.progressive_chunks - 1 and layer.inputs.chunk_bias is not None
        layer.forward("early")
        assert layer.verify()["pass"]
        first = _revealed_prefix(layer, c)
        ids_before = layer.expert_ids.clone()
        cut = layer.cfg.chunk_offsets[c + 1]
        g = torch.Generator(device="cpu").manual_seed(99)
        host = layer.inputs.tokens.cpu().clone()
        host[cut:] = torch.randn(host[cut:].shape, generator=g).to(host.dtype)
        layer.inputs.chunk_bias[c + 1:] += (torch.randn(layer.inputs.chunk_bias[c + 1:].shape, generator=g) * 3.0
                                            ).to(layer.inputs.chunk_bias.device)
        layer.load_tokens_(host.pin_memory())
        layer.forward("early")
        assert layer.verify()["pass"]
        second = _revealed_prefix(layer, c)
        assert torch.equal(first["ids"], second["ids"]) and torch.equal(first["gates"], second["gates"])
        assert torch.equal(first["log"], second["log"])
        for (m1, f1), (m2, f2) in zip(first["rows"], second["rows"]):
            assert torch.equal(m1, m2) and torch.equal(f1, f2)
        assert not torch.equal(ids_before[cut:], layer.expert_ids[cut:])  # the future did change
    finally:
        layer.close()


def test_peer_counters_count_one_call():
    """The device traffic counters behind PeerChannel.counters: one call on
    one rank puts every descriptor to itself once, with its rows' bytes, one
    ready signal per descriptor, one wait per descriptor, and returns every
    (token, choice) row once."""
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(_small("fp32", "gelu", 2), timeout_s=5.0)
    try:
        layer.forward("early")
        torch.cuda.synchronize()
        cfg = layer.cfg
        c = layer.channel.peer_counters()[0]
        rows = cfg.tokens_per_rank * cfg.top_k
        fwd_row = cfg.hidden * 4 + 9 * 8 + 4 + 4
        assert c["put_calls"] == cfg.n_desc and c["signals"] == cfg.n_desc and c["waits"] == cfg.n_desc
        assert c["bytes_transferred"] == rows * fwd_row + 4 * cfg.experts * cfg.n_desc
        assert c["return_bytes"] == rows * (cfg.out_dim * 4 + 8 * 8) and c["return_signals"] == 1
        layer.forward("early")
        assert layer.channel.counters["put_calls"] == 2 * cfg.n_desc
    finally:
        layer.close()


@pytest.mark.parametrize("name,over", [
    ("full_tf32", dict(tokens_per_rank=2048, chunk_sizes=(256,) * 8)),
    ("skewed_bf16", dict(tokens_per_rank=2048, chunk_sizes=(128,) * 16)),
    ("deepseek_v2_lite", dict(tokens_per_rank=1024, chunk_sizes=(64,) * 16)),
])
def test_progressive_gemm1_matches_and_starts_early(name, over):
    """GEMM-1 CTA pairs that take 256-row tiles as descriptors arrive compute
    exactly the tiles of the whole-batch plan: the layer's output is
    bit-identical with progressive planning on and off, in both arms, eagerly
    and replayed from a graph; and GEMM-1's first tile starts before the
    front end has finished."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    cfg = preset(name, **over)
    outs = {}
    for prog in (False, True):
        layer = ProgressiveMoELayer(cfg, timeout_s=10.0, progressive=prog, trace=True)
        try:
            for arm in ("early", "delayed"):
                layer.forward(arm)
                rep = layer.verify()
                assert rep["pass"], (prog, arm, rep["violations"])
                outs[(prog, arm)] = layer.out.clone()
            layer.forward("early")
            evs = {e["kind"]: e for e in layer.trace_events()}
            if prog:
                assert evs["gemm1"]["start_ns"] < evs["frontend"]["end_ns"], evs
            layer.capture("early")
            layer.replay("early")
            torch.cuda.synchronize()
            assert layer.verify()["pass"]
            outs[(prog, "graph")] = layer.out.clone()
        finally:
            layer.close()
    for key in ("early", "delayed", "graph"):
        assert torch.equal(outs[(False, key)], outs[(True, key)]), key


@pytest.mark.parametrize("name", ["r4_reference", "full_tf32", "skewed_bf16"])
def test_router_ring_matches_global_loads(name):
    """Routing token units out of the shared-memory ring (bulk copies issued
    ahead), and dispatching rows staged through that memory, give the same
    expert ids, gates and layer output as reading both from global memory."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    cfg = preset(name)
    if cfg.tokens_per_rank > 4096:
        n = cfg.chunks
        cfg = cfg.with_overrides(tokens_per_rank=4096, chunk_sizes=(4096 // n,) * n)
    res = {}
    for ring in (True, False):
        layer = ProgressiveMoELayer(cfg, timeout_s=5.0, router_ring=ring)
        try:
            for arm in ("early", "early"):
                layer.forward(arm)
                assert layer.verify()["pass"], ring
            res[ring] = (layer.expert_ids.clone(), layer.gates.clone(), layer.out.clone())
        finally:
            layer.close()
    for a, b in zip(res[True], res[False]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("name", ["r4_reference", "full_tf32"])
def test_dispatch_groups_match_shared_dispatch(name):
    """Descriptors dispatched by their own worker groups, side by side, leave the
    same rows, counts and layer output as every worker sharing every
    descriptor, in both arms."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    res = {}
    for groups in (True, False):
        layer = ProgressiveMoELayer(preset(name), timeout_s=5.0, dispatch_groups=groups)
        try:
            outs = []
            for arm in ("early", "delayed"):
                layer.forward(arm)
                assert layer.verify()["pass"], (groups, arm)
                outs.append(layer.out.clone())
            res[groups] = outs
        finally:
            layer.close()
    for a, b in zip(res[True], res[False]):
        assert torch.equal(a, b)


def test_prereleased_index_and_plain_dispatch_paths_both_run():
    """A worker whose descriptor is still held computes the descriptor's index
    part (prefix counts and ranks) before the release and then only copies;
    a worker whose descriptor is already released does both after it.  The
    early arm takes the first path for every descriptor still held when its
    workers reach it, the delayed arm always the second, and both arms leave
    the same verified output."""
    from revealaiccl_b200.bench.layer_probe import FE_CLOCK_SLOTS
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(preset("full_tf32"), timeout_s=5.0)
    try:
        sms = torch.cuda.get_device_properties(layer.device).multi_processor_count
        outs, indexed = {}, {}
        for arm in ("early", "delayed"):
            layer.tensors["fe_clock"] = torch.zeros(sms * FE_CLOCK_SLOTS, dtype=torch.int64, device=layer.device)
            layer.forward(arm)
            assert layer.verify()["pass"], arm
            stamps = layer.tensors["fe_clock"].cpu().view(sms, FE_CLOCK_SLOTS)[1:, 23]
            ran = stamps[stamps > 0] - 1  # descriptors indexed before release, per dispatching worker
            indexed[arm] = (int(ran.sum()), int((ran == 0).sum()), int(ran.numel()))
            outs[arm] = layer.out.clone()
        assert indexed["early"][0] > 0, indexed
        assert indexed["delayed"][0] == 0 and indexed["delayed"][2] > 0, indexed
        assert torch.equal(outs["early"], outs["delayed"])
    finally:
        layer.close()


TC_SHAPES = {
    "skewed_bf16": dict(tokens_per_rank=2048, chunk_sizes=(128,) * 16),
    "deepseek_v2_lite": dict(tokens_per_rank=2048, chunk_sizes=(128,) * 16),
    "mixtral_8x7b": dict(tokens_per_rank=1024, chunk_sizes=(96,) * 8 + (128, 96, 32) + (0,) * 21),
}


@pytest.mark.parametrize("name", sorted(TC_SHAPES))
def test_tensor_core_router_matches_warp_router(name):
    """bf16 batches route 128-token units on the tensor cores (tcgen05 MMA fed
    by TMA, accumulator in TMEM).  Against the warp router (CUDA-core dot
    products) the choices agree wherever the top-k is not a near tie, the gates
    agree to fp32 rounding, both pass the fail-closed checker against the fp32
    oracle, and a streamed end-to-end call routes exactly like a resident one
    (ragged and empty chunks included)."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    cfg = preset(name, **TC_SHAPES[name])
    res = {}
    for tc in (True, False):
        layer = ProgressiveMoELayer(cfg, timeout_s=5.0, router_tc=tc)
        try:
            layer.forward("early")
            assert layer.verify()["pass"], tc
            assert layer.runner.router_tc_used() == tc
            ids, gates, out = layer.expert_ids.clone(), layer.gates.clone(), layer.out.clone()
            layer.forward("delayed")
            assert layer.verify()["pass"] and torch.equal(out, layer.out)
            if tc:  # streamed end to end: the same routing as the resident call
                host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
                host_in.copy_(layer.inputs.tokens.cpu())
                host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
                layer(host_in, host_out, arm="early")
                torch.cuda.synchronize()
                assert layer.runner.router_tc_used()
                assert torch.equal(layer.expert_ids, ids) and torch.equal(layer.gates, gates)
                assert torch.equal(host_out, out.cpu())
            res[tc] = (ids, gates)
        finally:
            layer.close()
    (ia, ga), (ib, gb) = res[True], res[False]
    same = (ia == ib).all(dim=1)
    assert same.float().mean() > 0.99
    torch.testing.assert_close(ga[same], gb[same], atol=1e-5, rtol=1e-4)


def test_gemm1_split_k_matches_unsplit():
    """R4's GEMM-1 (2048 -> 32, 32 row tiles) splits K over otherwise idle SMs:
    each split stores a partial tile, the tile's last split adds them in split
    order.  The split ran (each tile's ticket counted its splits), the layer
    passes the checker, GEMM-1's activations agree with the unsplit GEMM's to
    fp32 rounding (only the order of the fp32 additions differs), the layer
    outputs agree within the tf32 tolerance (GEMM-2 rounds its inputs to tf32,
    so a last-bit change of an activation can move an output by ~1e-3), and
    results repeat bit for bit across calls and arms."""
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    cfg = preset("r4_reference")
    outs, tickets, hidden = {}, {}, {}
    for ks in (True, False):
        layer = ProgressiveMoELayer(cfg, timeout_s=5.0, gemm_ksplit=ks)
        try:
            layer.tensors["h"].zero_()  # rows GEMM-1 does not write stay equal in both layers
            layer.forward("early")
            assert layer.verify()["pass"], ks
            first = layer.out.clone()
            base = cfg.chunks * (1 + cfg.experts)
            tickets[ks] = layer.tensors["chunk_words"][base:].cpu()
            hidden[ks] = layer.tensors["h"].clone()
            layer.forward("delayed")
            assert layer.verify()["pass"] and torch.equal(first, layer.out)
            outs[ks] = first
        finally:
            layer.close()
    assert int(tickets[True].max()) > 1 and int(tickets[False].abs().sum()) == 0
    torch.testing.assert_close(hidden[True], hidden[False], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(outs[True], outs[False], atol=5e-3, rtol=5e-3)
