"""GPU: the routed MoE block (quantr_moe_dev / quantr_moe_layer) against the
oracle's per-token restatement of src/runtime.c:202-269 (qo_moe_token).

Routing (selected experts, in order) must be identical.  The expert GEMVs are
bit-exact, and softmax and silu evaluate expf exactly as the C library does
(csrc/libm_ref.cuh), so the renormalised weights and the block output must be
bit-identical to the oracle; the north-star bound (1e-5 rel / 1e-6 abs per
element) is asserted as well.
"""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


class Experts:
    """E packed matrices of one projection, contiguous like the merged
    *_exps tensors (src/model.c:409-419)."""

    def __init__(self, rng, type_, E, n, d, host=None):
        self.type, self.n, self.d, self.E = type_, n, d, E
        if host is None:
            host = np.stack([synth.matrix(rng, type_, n, d) for _ in range(E)])
        self.host = np.ascontiguousarray(host)
        self.stride = self.host[0].nbytes
        self.dev = _dev(self.host.reshape(-1))

    def weights(self, qr):
        return qr.ExpertWeights(self.dev.data_ptr(), self.stride, None, self.type)


def make_case(seed, T, E, k, dim, hidden, t1, t3, t2, router=False):
    rng = synth.rng_for(seed)
    c = {"T": T, "E": E, "k": k, "dim": dim, "hidden": hidden}
    c["w1"] = Experts(rng, t1, E, hidden, dim)
    c["w3"] = Experts(rng, t3, E, hidden, dim)
    c["w2"] = Experts(rng, t2, E, dim, hidden)
    c["xb"] = synth.activations(rng, T, dim)
    if router:
        c["router"] = (rng.standard_normal((E, dim), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
        c["logits"] = None
    else:
        c["router"] = None
        c["logits"] = rng.standard_normal((T, E), dtype=np.float32)
    return c


def oracle_case(orc, c):
    outs, sels, wts = [], [], []
    for t in range(c["T"]):
        o, s, w = orc.moe_token(c["xb"][t], c["E"], c["k"], c["w1"].host, c["w1"].type, c["w1"].stride,
                                c["w3"].host, c["w3"].type, c["w3"].stride, c["w2"].host, c["w2"].type,
                                c["w2"].stride, c["dim"], c["hidden"], router=c["router"],
                                logits=None if c["logits"] is None else c["logits"][t])
        outs.append(o)
        sels.append(s)
        wts.append(w)
    return np.stack(outs), np.stack(sels), np.stack(wts)


def run_dev(qr, c, w1=None, w3=None, w2=None):
    T, E, k, dim, hidden = c["T"], c["E"], c["k"], c["dim"], c["hidden"]
    xb = _dev(c["xb"])
    out = torch.full((T, dim), float("nan"), device="cuda")
    sel = torch.full((T, k), -7, dtype=torch.int32, device="cuda")
    wts = torch.full((T, k), float("nan"), device="cuda")
    ws_bytes = qr.moe_workspace_bytes(T, E, k, dim, hidden)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    router = None if c["router"] is None else _dev(c["router"])
    logits = None if c["logits"] is None else _dev(c["logits"])
    qr.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, E, k, w1 or c["w1"].weights(qr),
               w3 or c["w3"].weights(qr), w2 or c["w2"].weights(qr), dim, hidden, ws.data_ptr(), ws_bytes,
               router=None if router is None else router.data_ptr(),
               logits=None if logits is None else logits.data_ptr(), ldl=E, sel=sel.data_ptr(), wts=wts.data_ptr(),
               stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy(), sel.cpu().numpy(), wts.cpu().numpy()


def ulp_diff(a, b):
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


RTOL, ATOL = 1e-5, 1e-6  # the north-star bound, asserted per element


def check(got, want):
    """Routing identical, renormalised weights and block outputs bit-identical
    (the device evaluates expf exactly as the C library does), and the
    per-element north-star bound asserted on top."""
    go, gs, gw = got
    wo, ws, ww = want
    np.testing.assert_array_equal(gs, ws)
    assert ulp_diff(gw, ww).max() == 0, "renormalised weights differ"
    assert np.all(np.isfinite(go))
    assert np.all(np.abs(go - wo) <= ATOL + RTOL * np.abs(wo)), float(np.abs(go - wo).max())
    exact = float(np.mean(go.view(np.uint32) == wo.view(np.uint32)))
    assert exact == 1.0, f"only {exact:.6f} of the outputs are bit-identical"
    return exact


def test_moe_small_logits(qr_gpu, orc):
    c = make_case(1, T=7, E=8, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))
    assert qr_gpu.device_status() == 0


def test_moe_router_weights(qr_gpu, orc):
    """F32 router GEMV on the device (matmul_ref order) feeding the routing."""
    c = make_case(2, T=9, E=16, k=4, dim=768, hidden=512, t1=Q4_K, t3=Q4_K, t2=Q4_K, router=True)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))


def test_moe_c4_layer(qr_gpu, orc):
    """Qwen1.5-MoE routed experts: E=60, top-4, I=1408 (gate/up Q5_K 8 SB,
    down Q6_K with the 128-column tail ignored), hidden 2048, 64 tokens."""
    c = make_case(3, T=64, E=60, k=4, dim=2048, hidden=1408, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    exact = check(run_dev(qr_gpu, c), oracle_case(orc, c))
    print(f"c4 bit-identical fraction {exact:.6f}")


def test_moe_c4_layer_with_shared_expert(qr_gpu, orc):
    """BASELINE config c4 complete: the routed experts (60 of 1408, top-4,
    gate/up Q5_K, down Q6_K) plus the shared expert of 5632 with its sigmoid
    gate (quantr_moe_shared_dev), 64 tokens; bit-identical to the oracle's
    routed block followed by qo_shared_expert."""
    c = make_case(13, T=64, E=60, k=4, dim=2048, hidden=1408, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    rng = synth.rng_for(14)
    sh = 5632
    w1s, w3s = synth.matrix(rng, Q5_K, sh, 2048), synth.matrix(rng, Q5_K, sh, 2048)
    w2s = synth.matrix(rng, Q6_K, 2048, sh)
    gate = (rng.standard_normal(2048, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    T, dim = c["T"], c["dim"]
    xb = _dev(c["xb"])
    out = torch.full((T, dim), float("nan"), device="cuda")
    ws_bytes = qr_gpu.moe_workspace_bytes(T, c["E"], c["k"], dim, c["hidden"])
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    lg = _dev(c["logits"])
    d1, d3, d2, dg = _dev(w1s), _dev(w3s), _dev(w2s), _dev(gate)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the second call reuses the plans of the first
        qr_gpu.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, c["E"], c["k"], c["w1"].weights(qr_gpu),
                       c["w3"].weights(qr_gpu), c["w2"].weights(qr_gpu), dim, c["hidden"], ws.data_ptr(), ws_bytes,
                       logits=lg.data_ptr(), ldl=c["E"], stream=stream)
        qr_gpu.moe_shared_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, dg.data_ptr(), d1.data_ptr(), Q5_K,
                              d3.data_ptr(), Q5_K, d2.data_ptr(), Q6_K, dim, sh, stream)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        want, _, _ = oracle_case(orc, c)
        want = np.array(want, np.float32)
        for t in range(T):
            orc.shared_expert(want[t], c["xb"][t], gate, w1s, Q5_K, w3s, Q5_K, w2s, Q6_K, dim, sh)
        assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert qr_gpu.device_status() == 0


def test_moe_c5_layer(qr_gpu, orc):
    """Qwen3-30B-A3B experts: E=128, top-8, I=768 (3 SB), all Q4_K."""
    c = make_case(4, T=16, E=128, k=8, dim=2048, hidden=768, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))


def test_moe_mixed_types_and_ragged_hidden(qr_gpu, orc):
    """W1/W3 of different types (two grouped launches), a hidden size that is
    not a multiple of 32 (Q8_0 ignores the tail), Q8_0 down projection."""
    c = make_case(5, T=5, E=6, k=3, dim=256, hidden=200, t1=Q8_0, t3=Q4_K, t2=Q8_0)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))


def test_moe_hot_expert_many_passes(qr_gpu, orc):
    """Every token picks expert 3 first: its pair list is longer than one pass
    over the staged weight tile."""
    c = make_case(6, T=40, E=10, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    c["logits"][:, 3] += 8.0
    got = run_dev(qr_gpu, c)
    assert np.all(got[1][:, 0] == 3)
    check(got, oracle_case(orc, c))


def test_moe_ties_pick_lowest_index(qr_gpu, orc):
    c = make_case(7, T=3, E=12, k=4, dim=256, hidden=256, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    c["logits"][:] = 0.5
    got = run_dev(qr_gpu, c)
    assert np.all(got[1] == np.arange(4)[None, :])
    check(got, oracle_case(orc, c))


def test_moe_single_expert(qr_gpu, orc):
    c = make_case(8, T=4, E=1, k=1, dim=256, hidden=256, t1=Q6_K, t3=Q6_K, t2=Q6_K)
    got = run_dev(qr_gpu, c)
    assert np.all(got[1] == 0) and np.all(got[2] == 1.0)
    check(got, oracle_case(orc, c))


def test_moe_nan_logits_flag_routing_error(qr_gpu, orc):
    """A token with a NaN logit has no finite probabilities: the reference
    would index router_logits[-1]; here it gets no experts, out = 0, and the
    device status reports QUANTR_ERR_ROUTING.  Other tokens are unaffected."""
    c = make_case(9, T=4, E=8, k=2, dim=256, hidden=256, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    c["logits"][2, 5] = np.nan
    got_o, got_s, got_w = run_dev(qr_gpu, c)
    assert qr_gpu.device_status() == 9  # QUANTR_ERR_ROUTING (and reset)
    assert np.all(got_s[2] == -1) and np.all(got_o[2] == 0.0)
    keep = [0, 1, 3]
    c2 = dict(c)
    c2["T"] = 3
    c2["xb"] = c["xb"][keep]
    c2["logits"] = c["logits"][keep]
    check((got_o[keep], got_s[keep], got_w[keep]), oracle_case(orc, c2))
    assert qr_gpu.device_status() == 0


def test_moe_pointer_table(qr_gpu, orc):
    """Experts in separate allocations, addressed through a device table of
    pointers (the per-expert tensors of src/model.c:421-435)."""
    c = make_case(10, T=6, E=5, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    keep = []

    def tabled(ex):
        bufs = [_dev(ex.host[e]) for e in range(ex.E)]
        keep.extend(bufs)
        tab = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
        keep.append(tab)
        return qr_gpu.ExpertWeights(0, 0, tab.data_ptr(), ex.type)

    got = run_dev(qr_gpu, c, tabled(c["w1"]), tabled(c["w3"]), tabled(c["w2"]))
    check(got, oracle_case(orc, c))


def test_moe_rejects_bad_args(qr_gpu):
    c = make_case(11, T=2, E=4, k=2, dim=256, hidden=256, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    out = torch.zeros(2, 256, device="cuda")
    xb = _dev(c["xb"])
    lg = _dev(c["logits"])
    ws_bytes = qr_gpu.moe_workspace_bytes(2, 4, 2, 256, 256)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    w1, w3, w2 = c["w1"].weights(qr_gpu), c["w3"].weights(qr_gpu), c["w2"].weights(qr_gpu)
    for bad, code in [(dict(k=5), 3), (dict(k=0), 3), (dict(k=17, E=20), 3), (dict(E=300), 3),
                      (dict(ws_bytes=ws_bytes - 256), 8)]:
        a = dict(E=4, k=2, ws_bytes=ws_bytes)
        a.update(bad)
        with pytest.raises(qr_gpu.QuantrError) as ei:
            qr_gpu.moe_dev(out.data_ptr(), 256, xb.data_ptr(), 256, 2, a["E"], a["k"], w1, w3, w2, 256, 256,
                           ws.data_ptr(), a["ws_bytes"], logits=lg.data_ptr(), ldl=a["E"])
        assert ei.value.code == code, bad
    f32 = qr_gpu.ExpertWeights(c["w1"].dev.data_ptr(), c["w1"].stride, None, 0)
    with pytest.raises(qr_gpu.QuantrError) as ei:
        qr_gpu.moe_dev(out.data_ptr(), 256, xb.data_ptr(), 256, 2, 4, 2, f32, w3, w2, 256, 256, ws.data_ptr(),
                       ws_bytes, logits=lg.data_ptr(), ldl=4)
    assert ei.value.code == 4


def test_moe_layer_host_api(qr_gpu, orc):
    """quantr_moe_layer: host arrays of expert pointers into registered
    weights, as the reference's runtime holds them (w->expert_w1[l][e])."""
    c = make_case(12, T=5, E=6, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K, router=True)
    want = oracle_case(orc, c)
    mats = [c["w1"].host, c["w3"].host, c["w2"].host]
    for m in mats:
        qr_gpu.register_weights(m)
    try:
        got_o, got_s, got_w, rc = qr_gpu.moe_layer(c["xb"], 6, 2, list(mats[0]), Q5_K, list(mats[1]), Q5_K,
                                                   list(mats[2]), Q6_K, 512, 256, router=c["router"])
        assert rc == 0
        check((got_o, got_s, got_w), want)
        # Experts listed out of order: not evenly spaced, so a pointer table
        # is used; the oracle sees the same permuted experts and router rows.
        inv = np.array([3, 1, 0, 5, 2, 4])
        cp = dict(c)
        for key in ("w1", "w3", "w2"):
            ex = c[key]
            cp[key] = Experts(None, ex.type, ex.E, ex.n, ex.d, host=ex.host[inv])
        cp["router"] = np.ascontiguousarray(c["router"][inv])
        got2 = qr_gpu.moe_layer(c["xb"], 6, 2, [mats[0][i] for i in inv], Q5_K, [mats[1][i] for i in inv], Q5_K,
                                [mats[2][i] for i in inv], Q6_K, 512, 256, router=cp["router"])
        assert got2[3] == 0
        check(got2[:3], oracle_case(orc, cp))
    finally:
        for m in mats:
            qr_gpu.unregister_weights(m)
    # Unregistered expert weights are refused and out is zeroed.
    o, s, w, rc = qr_gpu.moe_layer(c["xb"], 6, 2, list(mats[0]), Q5_K, list(mats[1]), Q5_K, list(mats[2]), Q6_K,
                                   512, 256, router=c["router"])
    assert rc == 10 and np.all(o == 0.0)


@pytest.mark.parametrize("T", [9, 56])
def test_moe_stages_emulate_expert_parallel(qr_gpu, orc, T):
    """route once, run the experts stage on two disjoint expert ranges into
    zeroed buffers (what two expert-parallel ranks compute), add them (each row
    has one non-zero contributor, so the sum is exact), combine: bit-identical
    to quantr_moe_dev.  T = 56 takes the tensor-core experts stage."""
    c = make_case(13, T=T, E=10, k=3, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    full = run_dev(qr_gpu, c)
    E, k, dim, hidden = 10, 3, 512, 256
    s = torch.cuda.current_stream().cuda_stream
    xb = _dev(c["xb"])
    lg = _dev(c["logits"])
    ws_bytes = qr_gpu.moe_workspace_bytes(T, E, k, dim, hidden)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    sel = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    qr_gpu.moe_route_dev(sel.data_ptr(), wts.data_ptr(), xb.data_ptr(), dim, T, E, k, dim, ws.data_ptr(), ws_bytes,
                         logits=lg.data_ptr(), ldl=E, stream=s)
    parts = []
    for e0, e1 in ((0, 4), (4, 10)):
        o = torch.zeros(T * k, dim, device="cuda")
        ws_i = torch.empty(qr_gpu.moe_workspace_bytes(T, e1 - e0, k, dim, hidden), dtype=torch.uint8, device="cuda")
        ew = []
        for key in ("w1", "w3", "w2"):
            ex = c[key]
            ew.append(qr_gpu.ExpertWeights(ex.dev.data_ptr() + e0 * ex.stride, ex.stride, None, ex.type))
        qr_gpu.moe_experts_dev(o.data_ptr(), xb.data_ptr(), dim, T, sel.data_ptr(), k, e0, e1 - e0, *ew, dim, hidden,
                               ws_i.data_ptr(), ws_i.numel(), stream=s)
        parts.append(o)
    o = parts[0] + parts[1]
    out = torch.empty(T, dim, device="cuda")
    qr_gpu.moe_combine_dev(out.data_ptr(), dim, o.data_ptr(), sel.data_ptr(), wts.data_ptr(), T, k, dim, stream=s)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(sel.cpu().numpy(), full[1])
    np.testing.assert_array_equal(wts.cpu().numpy().view(np.uint32), full[2].view(np.uint32))
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), full[0].view(np.uint32))


# Tensor-core experts stage (T >= 16 tokens: gathered tcgen05 jobs over each
# expert's pairs) on the cases above that shape it differently.

def test_moe_tc_mixed_types(qr_gpu, orc):
    """W1 Q4_K with W3 Q8_0 (different element order and unit count: W3 gets
    operand tiles of its own), Q6_K down projection over a ragged hidden."""
    c = make_case(21, T=48, E=6, k=3, dim=512, hidden=320, t1=Q4_K, t3=Q8_0, t2=Q6_K)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))


def test_moe_tc_hot_expert_four_passes(qr_gpu, orc):
    """All 64 tokens pick expert 3 first: its job runs four 16-pair passes."""
    c = make_case(22, T=64, E=10, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    c["logits"][:, 3] += 8.0
    got = run_dev(qr_gpu, c)
    assert np.all(got[1][:, 0] == 3)
    check(got, oracle_case(orc, c))


def test_moe_tc_pointer_table_and_idle_experts(qr_gpu, orc):
    """Experts addressed through a device pointer table (read once when the
    launch plan is built); two experts nobody picks are skipped."""
    c = make_case(23, T=48, E=8, k=2, dim=512, hidden=256, t1=Q5_K, t3=Q5_K, t2=Q6_K)
    c["logits"][:, 6:] -= 50.0
    keep = []

    def tabled(ex):
        bufs = [_dev(ex.host[e]) for e in range(ex.E)]
        keep.extend(bufs)
        tab = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
        keep.append(tab)
        return qr_gpu.ExpertWeights(0, 0, tab.data_ptr(), ex.type)

    got = run_dev(qr_gpu, c, tabled(c["w1"]), tabled(c["w3"]), tabled(c["w2"]))
    assert not np.isin(got[1], [6, 7]).any()
    check(got, oracle_case(orc, c))
    got2 = run_dev(qr_gpu, c, tabled(c["w1"]), tabled(c["w3"]), tabled(c["w2"]))  # new tables: a new plan
    np.testing.assert_array_equal(got2[0].view(np.uint32), got[0].view(np.uint32))


def test_moe_tc_repeat_call_new_tokens(qr_gpu, orc):
    """The cached launch plan reused with new inputs in the same buffers."""
    c = make_case(24, T=64, E=8, k=2, dim=512, hidden=256, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    T, E, k, dim, hidden = 64, 8, 2, 512, 256
    xb = _dev(c["xb"])
    lg = _dev(c["logits"])
    out = torch.empty(T, dim, device="cuda")
    ws_bytes = qr_gpu.moe_workspace_bytes(T, E, k, dim, hidden)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    w = [c[key].weights(qr_gpu) for key in ("w1", "w3", "w2")]
    s = torch.cuda.current_stream().cuda_stream
    rng = synth.rng_for(25)
    for it in range(2):
        if it:
            c["xb"] = synth.activations(rng, T, dim)
            c["logits"] = rng.standard_normal((T, E), dtype=np.float32)
            xb.copy_(torch.from_numpy(c["xb"]))
            lg.copy_(torch.from_numpy(c["logits"]))
        sel = torch.empty(T, k, dtype=torch.int32, device="cuda")
        wts = torch.empty(T, k, device="cuda")
        qr_gpu.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, E, k, *w, dim, hidden, ws.data_ptr(), ws_bytes,
                       logits=lg.data_ptr(), ldl=E, sel=sel.data_ptr(), wts=wts.data_ptr(), stream=s)
        torch.cuda.synchronize()
        check((out.cpu().numpy(), sel.cpu().numpy(), wts.cpu().numpy()), oracle_case(orc, c))


@pytest.mark.parametrize("T,k", [(200, 2), (512, 1)])
def test_moe_tc_more_tokens_than_a_job(qr_gpu, orc, T, k):
    """More tokens than one tensor-core job holds (64): the experts stage
    still runs as gathered 16-pair passes per expert (the expert-parallel
    owner's case: its received pairs are 512 one-slot tokens at the c5
    shape)."""
    c = make_case(31 + T, T=T, E=12, k=k, dim=512, hidden=256, t1=Q4_K, t3=Q4_K, t2=Q4_K)
    check(run_dev(qr_gpu, c), oracle_case(orc, c))
