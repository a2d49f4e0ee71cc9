"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed
(NCCL over NVLink/NVSwitch) for the exchange steps each form has.

Row-sharded (tensor-parallel) GEMV.  Every packed block lies inside one row
(src/quant.c:491-492), so a contiguous range of rows is a contiguous byte range
of the packed matrix.  Rank r of P owns rows [r*np, min(n, (r+1)*np)) with
np = ceil(n/P); x is replicated and every rank quantizes it with the same
kernel, so the activation blocks are bit-identical on every rank, and each
output row is exactly what one GPU computes for it.  One all-gather of the
np-row shards assembles out.

Expert-parallel MoE (src/runtime.c:202-269), tokens and experts both split.
Rank r holds its own tokens and owns experts [E*r/P, E*(r+1)/P).  Each rank
routes its tokens (the router is per token) and orders its (token, slot)
pairs by destination on the device, then:
  1. counts: every rank tells every other how many (token, slot) pairs it
     will send it (all_to_all_single of P counts);
  2. dispatch: each pair's activation row goes to the owner of its expert as
     the reference's own Q8_0 blocks (quantize_row_q8_0 of xb, 34 bytes per
     32 elements, 3.8x fewer bytes than fp32) with the expert id
     (all_to_all_single).  The reference quantizes the same xb identically
     for every expert call (src/runtime.c:252-253 -> src/quant.c:474), and
     re-quantizing the exact dequantization of such blocks reproduces them,
     so the owner's GEMVs see the very activations one GPU would;
  3. the owner runs its experts on the received pairs (one slot each);
  4. return: every pair's output row goes back to its token's rank
     (all_to_all_single), which combines in selection order
     (src/runtime.c:262-264).
Every per-pair output is computed by the same kernels on the same bytes as
on one GPU, so the block output is bit-identical to the unsharded one.

Compute goes through a backend object with the library's stage calls
(`CudaBackend`, the product path on the C ABI); the host logic here (shard
ranges, padding, reassembly, dispatch plans, exchanges, combine order) is
backend-agnostic.
"""
import numpy as np
import torch
import torch.distributed as dist

import quantr


def row_range(n, rank, world):
    """Rows [r0, r1) of rank `rank` and the padded shard height np."""
    npad = -(-n // world)
    r0 = min(n, rank * npad)
    return r0, min(n, r0 + npad), npad


def expert_range(E, rank, world):
    """Experts [e0, e1) of rank `rank`."""
    return E * rank // world, E * (rank + 1) // world


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


class CudaBackend:
    """The library's device calls on torch device buffers (current device)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self._ws = None

    def _workspace(self, nbytes):
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._ws

    def stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def upload(self, host_bytes):
        # 16 spare bytes keep every bulk-copy window of the last row in bounds.
        t = torch.zeros(host_bytes.nbytes + 16, dtype=torch.uint8, device=self.device)
        t[:host_bytes.nbytes].copy_(torch.from_numpy(np.ascontiguousarray(host_bytes).reshape(-1)))
        return t

    def zeros(self, *shape):
        return torch.zeros(*shape, dtype=torch.float32, device=self.device)

    def gemv(self, out, ldo, x, w, type_, n, d):
        B = x.shape[0]
        need = quantr.workspace_bytes(d, B)
        ws = self._workspace(need)
        quantr.gemv_dev(out.data_ptr(), ldo, x.data_ptr(), x.stride(0), w.data_ptr(), type_, n, d, B,
                        ws.data_ptr(), ws.numel(), self.stream())

    def route(self, xb, E, k, router=None, logits=None):
        T, dim = xb.shape
        sel = torch.empty(T, k, dtype=torch.int32, device=self.device)
        wts = torch.empty(T, k, dtype=torch.float32, device=self.device)
        ws = self._workspace(quantr.moe_workspace_bytes(T, E, k, dim, 1))
        quantr.moe_route_dev(sel.data_ptr(), wts.data_ptr(), xb.data_ptr(), xb.stride(0), T, E, k, dim,
                             ws.data_ptr(), ws.numel(), router=None if router is None else router.data_ptr(),
                             logits=None if logits is None else logits.data_ptr(),
                             ldl=0 if logits is None else logits.stride(0), stream=self.stream())
        return sel, wts

    def experts(self, o, xb, sel, e0, El, mats, dim, hidden):
        T, k = sel.shape
        ws = self._workspace(quantr.moe_workspace_bytes(T, El, k, dim, hidden))
        ew = [quantr.ExpertWeights(t.data_ptr(), stride, None, type_) for t, stride, type_ in mats]
        quantr.moe_experts_dev(o.data_ptr(), xb.data_ptr(), xb.stride(0), T, sel.data_ptr(), k, e0, El, ew[0], ew[1],
                               ew[2], dim, hidden, ws.data_ptr(), ws.numel(), stream=self.stream())

    def combine(self, o, sel, wts, dim):
        T, k = sel.shape
        out = torch.empty(T, dim, dtype=torch.float32, device=self.device)
        quantr.moe_combine_dev(out.data_ptr(), dim, o.data_ptr(), sel.data_ptr(), wts.data_ptr(), T, k, dim,
                               stream=self.stream())
        return out

    def quantize_q8_0(self, x):
        """T x d fp32 -> T x (d/32*34) uint8 packed block_q8_0 rows."""
        T, d = x.shape
        y = torch.empty(T, (d // 32) * 34, dtype=torch.uint8, device=self.device)
        if T:
            quantr.quantize_q8_0_dev(y.data_ptr(), x.data_ptr(), x.stride(0), d, T, self.stream())
        return y

    def dequantize_q8_0(self, y, d):
        """Packed block_q8_0 rows -> T x d fp32 (dequantize_row per row)."""
        T = y.shape[0]
        x = torch.zeros(T, d, dtype=torch.float32, device=self.device)
        if T:
            quantr.dequantize_rows_dev(x.data_ptr(), d, y.data_ptr(), y.stride(0), 8, d, T, self.stream())
        return x


class RowShardedGemv:
    """out = W.x for a packed n x d matrix whose rows are split over the group.

    w_host: uint8[n, row_bytes] (the whole packed matrix as loaded; each rank
    uploads only its rows).  __call__(x) takes x as B x d on this rank's
    device (replicated) and returns the full B x n output on every rank."""

    def __init__(self, w_host, type_, n, d, backend, group=None):
        self.world, self.rank = _world(group)
        self.group, self.backend = group, backend
        self.type, self.n, self.d = type_, n, d
        self.r0, self.r1, self.npad = row_range(n, self.rank, self.world)
        rb = quantr.row_bytes(type_, d)
        w_host = np.asarray(w_host, np.uint8).reshape(n, rb) if n * rb else np.zeros((n, 0), np.uint8)
        self.w = backend.upload(w_host[self.r0:self.r1])

        self._bufs = {}

    def __call__(self, x):
        # Buffers per batch size, allocated once (a call allocates nothing, so
        # it can be captured in a CUDA graph with its all-gather).
        B = x.shape[0]
        if B not in self._bufs:
            self._bufs[B] = (self.backend.zeros(B, self.npad), self.backend.zeros(self.world * B * self.npad))
        local, gathered = self._bufs[B]
        if self.r1 > self.r0:
            self.backend.gemv(local, self.npad, x, self.w, self.type, self.r1 - self.r0, self.d)
        if self.world == 1:
            return local[:, :self.n]
        dist.all_gather_into_tensor(gathered, local.reshape(-1), group=self.group)
        if B == 1:
            return gathered.view(1, self.world * self.npad)[:, :self.n]
        full = gathered.view(self.world, B, self.npad).permute(1, 0, 2).reshape(B, self.world * self.npad)
        return full[:, :self.n]


class ExpertShardedMoE:
    """The routed MoE block with tokens and experts split over the group.

    w1/w3: uint8[E, hidden, row_bytes(t, dim)], w2: uint8[E, dim,
    row_bytes(t2, hidden)] (the merged *_exps tensors, src/model.c:409-419);
    each rank uploads its experts only.  router: E x dim F32 on this rank's
    device, or None with logits given per call.  __call__(xb) takes THIS
    rank's tokens (T_r x dim) and returns (out, sel, wts) for them; `stats`
    then holds the pairs sent/received and the bytes each exchange moved."""

    def __init__(self, E, k, dim, hidden, w1, t1, w3, t3, w2, t2, backend, group=None, router=None):
        self.world, self.rank = _world(group)
        self.group, self.backend = group, backend
        self.E, self.k, self.dim, self.hidden = E, k, dim, hidden
        self.e0, self.e1 = expert_range(E, self.rank, self.world)
        self.router = router
        self.owner = torch.tensor([max(r for r in range(self.world) if expert_range(E, r, self.world)[0] <= e)
                                   for e in range(E)], dtype=torch.int64)
        self.mats = []
        for w, t in ((w1, t1), (w3, t3), (w2, t2)):
            w = np.asarray(w, np.uint8)
            local = w[self.e0:self.e1]
            stride = int(np.prod(w.shape[1:])) if w.ndim > 1 else 0
            self.mats.append((backend.upload(local), stride, t))
        self.stats = {}
        self._owner_dev = None

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def __call__(self, xb, logits=None):
        T, dim, k = xb.shape[0], self.dim, self.k
        be = self.backend
        sel, wts = be.route(xb, self.E, k, router=self.router, logits=logits)
        # Dispatch plan on the tokens' device: valid pairs ordered by
        # destination rank, then pair index (pairs without an expert go last).
        dev = xb.device
        if self._owner_dev is None or self._owner_dev.device != dev:
            self._owner_dev = self.owner.to(dev)
        selv = sel.reshape(-1).to(torch.int64)
        valid = selv >= 0
        dest = torch.where(valid, self._owner_dev[selv.clamp(min=0)], torch.full_like(selv, self.world))
        order = torch.argsort(dest * (T * k + 1) + torch.arange(T * k, device=dev))
        # 1. counts (NCCL takes device tensors only; gloo host ones); the one
        # value that comes back to the host is the pair counts, which size
        # the variable-length exchanges.
        send_counts = torch.bincount(dest, minlength=self.world + 1)[:self.world].to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        counts = torch.cat([send_counts, recv_counts]).tolist()
        sc, rc = counts[:self.world], counts[self.world:]
        pair = order[:sum(sc)]
        sel_h = selv
        n_send, n_recv = sum(sc), sum(rc)
        # 2. dispatch: Q8_0 rows of the pairs' tokens, and their expert ids.
        xq = be.quantize_q8_0(xb)
        tok = pair // k
        send_q = xq.index_select(0, tok) if n_send else xq[:0]
        recv_q = torch.empty(n_recv, xq.shape[1], dtype=torch.uint8, device=dev)
        self._a2a(recv_q, send_q, rc, sc)
        send_e = sel_h[pair].to(torch.int32)
        recv_e = torch.empty(n_recv, dtype=torch.int32, device=dev)
        self._a2a(recv_e, send_e, rc, sc)
        # 3. local experts on the received pairs (one slot each).
        o_recv = be.zeros(n_recv, dim)
        if n_recv and self.e1 > self.e0:
            be.experts(o_recv, be.dequantize_q8_0(recv_q, dim), recv_e.view(n_recv, 1), self.e0,
                       self.e1 - self.e0, self.mats, dim, self.hidden)
        # 4. outputs back to the tokens' ranks, then the combine.
        o_back = be.zeros(n_send, dim)
        self._a2a(o_back, o_recv, sc, rc)
        o = be.zeros(T * k, dim)
        if n_send:
            o.index_copy_(0, pair, o_back)
        self.stats = {"pairs_sent": n_send, "pairs_received": n_recv,
                      "dispatch_bytes": n_send * (xq.shape[1] + 4), "return_bytes": n_send * dim * 4}
        return be.combine(o, sel, wts, dim), sel, wts
