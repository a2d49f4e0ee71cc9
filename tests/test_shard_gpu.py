"""GPU, 2 ranks over NCCL: the row-sharded GEMV (all-gather) and the
expert-parallel MoE (tokens split, all-to-all dispatch of Q8_0 activations
and return of per-pair outputs) of quantr-in-c_b200/shard.py on real
devices.  The sharded GEMV must be bit-identical to the oracle; the sharded
MoE bit-identical to the one-GPU quantr_moe_dev result.  Skipped on boxes
with fewer than 2 GPUs (bench.py --gpus N runs the same forms on every
GPU count and reports their parity with one GPU)."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import synth  # noqa: E402

Q4_K, Q5_K, Q6_K, Q8_0 = 12, 13, 14, 8
WORLD = 2


def _case():
    rng = synth.rng_for(31)
    c = {"gemv": [(Q4_K, 4864, 896), (Q6_K, 1001, 2048), (Q8_0, 333, 4096)]}
    c["gemv_w"] = [synth.matrix(rng, t, n, d) for t, n, d in c["gemv"]]
    c["x"] = {d: synth.activations(rng, 2, d) for _, _, d in c["gemv"]}
    E, k, dim, hidden = 12, 4, 2048, 1408
    c["moe"] = (E, k, dim, hidden)
    c["w1"] = np.stack([synth.matrix(rng, Q5_K, hidden, dim) for _ in range(E)])
    c["w3"] = np.stack([synth.matrix(rng, Q5_K, hidden, dim) for _ in range(E)])
    c["w2"] = np.stack([synth.matrix(rng, Q6_K, dim, hidden) for _ in range(E)])
    c["xb"] = synth.activations(rng, 16, dim)
    c["logits"] = rng.standard_normal((16, E), dtype=np.float32)
    return c


def _rank(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import quantr
        import shard
        assert quantr.lib().quantr_gpu_init(rank) == 0
        be = shard.CudaBackend(dev)
        c = _case()
        res = {}
        for i, ((t, n, d), w) in enumerate(zip(c["gemv"], c["gemv_w"])):
            g = shard.RowShardedGemv(w, t, n, d, be)
            res[f"gemv{i}"] = g(torch.from_numpy(c["x"][d]).to(dev)).cpu().numpy()
        E, k, dim, hidden = c["moe"]
        m = shard.ExpertShardedMoE(E, k, dim, hidden, c["w1"], Q5_K, c["w3"], Q5_K, c["w2"], Q6_K, be)
        T = c["xb"].shape[0]
        t0, t1 = T * rank // world, T * (rank + 1) // world  # this rank's tokens
        out, sel, wts = m(torch.from_numpy(c["xb"][t0:t1]).to(dev),
                          logits=torch.from_numpy(c["logits"][t0:t1]).to(dev))
        torch.cuda.synchronize()
        parts = [None] * world
        dist.all_gather_object(parts, (out.cpu().numpy(), sel.cpu().numpy(), wts.cpu().numpy()))
        res["moe"] = np.concatenate([p[0] for p in parts])
        res["sel"] = np.concatenate([p[1] for p in parts])
        res["wts"] = np.concatenate([p[2] for p in parts])
        assert quantr.device_status(0) == 0
        dist.barrier()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_gemv_and_moe_nccl(tmp_path, orc):
    mp.spawn(_rank, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    c = _case()
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(WORLD)]
    for key in r[0].files:  # every rank holds the same full result
        np.testing.assert_array_equal(r[0][key].view(np.uint8), r[1][key].view(np.uint8), err_msg=key)
    for i, ((t, n, d), w) in enumerate(zip(c["gemv"], c["gemv_w"])):
        want = orc.matmul_q_fused_batch(c["x"][d], w, t, n, d)
        np.testing.assert_array_equal(r[0][f"gemv{i}"].view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
    # The one-GPU MoE on the same inputs.
    import quantr
    E, k, dim, hidden = c["moe"]
    T = c["xb"].shape[0]
    mats = [torch.from_numpy(np.ascontiguousarray(c[key]).reshape(-1)).cuda() for key in ("w1", "w3", "w2")]
    ew = [quantr.ExpertWeights(m.data_ptr(), c[key][0].nbytes, None, t)
          for m, key, t in zip(mats, ("w1", "w3", "w2"), (Q5_K, Q5_K, Q6_K))]
    xb, lg = torch.from_numpy(c["xb"]).cuda(), torch.from_numpy(c["logits"]).cuda()
    out = torch.empty(T, dim, device="cuda")
    wsb = quantr.moe_workspace_bytes(T, E, k, dim, hidden)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    quantr.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, E, k, *ew, dim, hidden, ws.data_ptr(), wsb,
                   logits=lg.data_ptr(), ldl=E, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r[0]["moe"].view(np.uint32), out.cpu().numpy().view(np.uint32))
