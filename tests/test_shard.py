"""CPU (gloo, world_size 2): the host logic of the multi-GPU forms in
quantr-in-c_b200/shard.py - shard ranges, padding, the all-gather reassembly of
row shards, the expert and token split, the all-to-all exchanges (counts, Q8_0
activation dispatch, per-pair output return) and the selection-order combine.

The compute runs on a CPU stand-in backend built from the oracle (test
infrastructure); the property checked is that the sharded result is
bit-identical to the same backend run unsharded (world_size 1).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import shard  # noqa: E402
import synth  # noqa: E402

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14


class CpuBackend:
    """Stage calls of shard.CudaBackend restated on the CPU with the oracle."""

    def __init__(self):
        import oracle
        self.orc = oracle.Oracle()

    def upload(self, host_bytes):
        return np.ascontiguousarray(host_bytes)

    def zeros(self, *shape):
        return torch.zeros(*shape, dtype=torch.float32)

    def gemv(self, out, ldo, x, w, type_, n, d):
        res = self.orc.matmul_q_fused_batch(x.numpy(), w.reshape(-1), type_, n, d)
        out[:, :n] = torch.from_numpy(np.asarray(res, np.float32).reshape(x.shape[0], n))

    def route(self, xb, E, k, router=None, logits=None):
        T = xb.shape[0]
        sel = np.empty((T, k), np.int32)
        wts = np.empty((T, k), np.float32)
        for t in range(T):
            lg = logits[t].numpy() if router is None else self.orc.matmul_f32(xb[t].numpy(), router, E, xb.shape[1])
            p = self.orc.softmax(lg)
            for s in range(k):
                arg = int(np.argmax(p))  # first maximum: the reference's strict '>' scan
                sel[t, s], wts[t, s] = arg, p[arg]
                p[arg] = np.float32(-1e9)
            tot = np.float32(0.0)
            for s in range(k):
                tot = np.float32(tot + wts[t, s])
            wts[t] = (wts[t] / tot).astype(np.float32)
        return torch.from_numpy(sel), torch.from_numpy(wts)

    def experts(self, o, xb, sel, e0, El, mats, dim, hidden):
        (w1, s1, t1), (w3, s3, t3), (w2, s2, t2) = mats
        flat = sel.numpy().reshape(-1)
        k = sel.shape[1]
        for p, e in enumerate(flat):
            if not (e0 <= e < e0 + El):
                continue
            le = e - e0
            x = xb[p // k].numpy()
            h1 = self.orc.matmul_q_fused(x, w1.reshape(-1)[le * s1:(le + 1) * s1], t1, hidden, dim)
            h3 = self.orc.matmul_q_fused(x, w3.reshape(-1)[le * s3:(le + 1) * s3], t3, hidden, dim)
            h1 = np.asarray(h1, np.float32)
            hb = (h1 / (np.float32(1.0) + np.exp(-h1)) * np.asarray(h3, np.float32)).astype(np.float32)
            o[p] = torch.from_numpy(np.asarray(
                self.orc.matmul_q_fused(hb, w2.reshape(-1)[le * s2:(le + 1) * s2], t2, dim, hidden), np.float32))

    def quantize_q8_0(self, x):
        xn = x.numpy()
        return torch.from_numpy(np.stack([self.orc.quantize_row_q8_0(r) for r in xn]) if len(xn)
                                else np.zeros((0, (x.shape[1] // 32) * 34), np.uint8))

    def dequantize_q8_0(self, y, d):
        yn = y.numpy()
        return torch.from_numpy(np.stack([self.orc.dequantize_row(r, Q8_0, d) for r in yn]).astype(np.float32)
                                if len(yn) else np.zeros((0, d), np.float32))

    def combine(self, o, sel, wts, dim):
        T, k = sel.shape
        out = np.zeros((T, dim), np.float32)
        on, sn, wn = o.numpy(), sel.numpy(), wts.numpy()
        for t in range(T):
            acc = np.zeros(dim, np.float32)
            for s in range(k):
                if sn[t, s] >= 0:
                    acc = (acc + on[t * k + s] * wn[t, s]).astype(np.float32)
            out[t] = acc
        return torch.from_numpy(out)


def _case(seed):
    rng = synth.rng_for(seed)
    c = {}
    c["gemv"] = [(Q4_K, 37, 512), (Q6_K, 5, 768), (Q8_0, 64, 96)]
    c["gemv_w"] = [synth.matrix(rng, t, n, d) for t, n, d in c["gemv"]]
    c["x"] = {d: synth.activations(rng, 3, d) for _, _, d in c["gemv"]}
    E, k, dim, hidden = 6, 2, 256, 256
    c["moe"] = (E, k, dim, hidden)
    c["w1"] = np.stack([synth.matrix(rng, Q5_K, hidden, dim) for _ in range(E)])
    c["w3"] = np.stack([synth.matrix(rng, Q5_K, hidden, dim) for _ in range(E)])
    c["w2"] = np.stack([synth.matrix(rng, Q6_K, dim, hidden) for _ in range(E)])
    c["xb"] = synth.activations(rng, 7, dim)
    c["logits"] = rng.standard_normal((7, E), dtype=np.float32)
    return c


def _run(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be = CpuBackend()
        c = _case(5)
        res = {}
        for i, ((t, n, d), w) in enumerate(zip(c["gemv"], c["gemv_w"])):
            g = shard.RowShardedGemv(w, t, n, d, be)
            res[f"gemv{i}"] = g(torch.from_numpy(c["x"][d])).numpy().copy()
        E, k, dim, hidden = c["moe"]
        m = shard.ExpertShardedMoE(E, k, dim, hidden, c["w1"], Q5_K, c["w3"], Q5_K, c["w2"], Q6_K, be)
        T = c["xb"].shape[0]
        t0, t1 = T * rank // world, T * (rank + 1) // world  # this rank's tokens
        out, sel, wts = m(torch.from_numpy(c["xb"][t0:t1]), logits=torch.from_numpy(c["logits"][t0:t1]))
        parts = [None] * world
        dist.all_gather_object(parts, (out.numpy(), sel.numpy(), wts.numpy(), m.stats))
        res["moe"] = np.concatenate([p[0] for p in parts])
        res["sel"] = np.concatenate([p[1] for p in parts])
        res["wts"] = np.concatenate([p[2] for p in parts])
        if rank == 0:
            np.savez(os.path.join(out_dir, f"w{world}.npz"), **res)
            sent = sum(p[3]["pairs_sent"] for p in parts)
            recv = sum(p[3]["pairs_received"] for p in parts)
            assert sent == recv == T * k, (sent, recv)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ranges_cover_rows_and_experts():
    for n in (1, 5, 37, 4864):
        for world in (1, 2, 3, 8):
            rows = [shard.row_range(n, r, world) for r in range(world)]
            assert rows[0][0] == 0 and rows[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
            assert all(r1 - r0 <= rows[0][2] for r0, r1, _ in rows)
    for E in (1, 7, 60, 128):
        for world in (1, 2, 4, 8):
            ex = [shard.expert_range(E, r, world) for r in range(world)]
            assert ex[0][0] == 0 and ex[-1][1] == E
            assert all(a[1] == b[0] for a, b in zip(ex, ex[1:]))


def test_sharded_equals_unsharded_gloo(tmp_path):
    for world in (1, 2):
        mp.spawn(_run, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    a = np.load(tmp_path / "w1.npz")
    b = np.load(tmp_path / "w2.npz")
    for key in a.files:
        np.testing.assert_array_equal(np.asarray(a[key]).view(np.uint8), np.asarray(b[key]).view(np.uint8),
                                      err_msg=key)
