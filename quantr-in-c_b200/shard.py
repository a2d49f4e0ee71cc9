"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed
(NCCL over NVLink/NVSwitch) for the one exchange step each form has.

Row-sharded (tensor-parallel) GEMV.  Every packed block lies inside one row
(src/quant.c:491-492), so a contiguous range of rows is a contiguous byte range
of the packed matrix.  Rank r of P owns rows [r*np, min(n, (r+1)*np)) with
np = ceil(n/P); x is replicated and every rank quantizes it with the same
kernel, so the activation blocks are bit-identical on every rank, and each
output row is exactly what one GPU computes for it.  One all-gather of the
np-row shards assembles out.

Expert-parallel MoE (src/runtime.c:202-269).  Rank r owns experts
[E*r/P, E*(r+1)/P).  Every rank routes every token with the same kernel on the
same inputs (identical sel/wts), runs its own experts on the (token, slot)
pairs routed to them, writing those rows of a zeroed (T*k) x dim buffer, and
one all-reduce (sum) assembles it: each row has exactly one non-zero
contributor and x + 0.0 == x, so the sum is exact whatever order the
collective adds in (a -0.0 row becomes +0.0, which the combine's
0.0f + o*ew cannot tell apart).  Every rank then combines in selection order.

Compute goes through a backend object with the library's stage calls
(`CudaBackend`, the product path on the C ABI); the host logic here (shard
ranges, padding, reassembly, exchange, combine order) is backend-agnostic.
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

    def __call__(self, x):
        B = x.shape[0]
        local = self.backend.zeros(B, self.npad)
        if self.r1 > self.r0:
            self.backend.gemv(local, self.npad, x, self.w, self.type, self.r1 - self.r0, self.d)
        gathered = self.backend.zeros(self.world * B * self.npad)
        dist.all_gather_into_tensor(gathered, local.reshape(-1), group=self.group)
        full = gathered.view(self.world, B, self.npad).permute(1, 0, 2).reshape(B, self.world * self.npad)
        return full[:, :self.n]


class ExpertShardedMoE:
    """The routed MoE block with experts split over the group.

    w1/w3: uint8[E, hidden, row_bytes(t, dim)], w2: uint8[E, dim,
    row_bytes(t2, hidden)] (the merged *_exps tensors, src/model.c:409-419);
    each rank uploads its experts only.  router: E x dim F32 on this rank's
    device, or None with logits given per call.  __call__ returns (out, sel,
    wts) on every rank."""

    def __init__(self, E, k, dim, hidden, w1, t1, w3, t3, w2, t2, backend, group=None, router=None):
        self.world, self.rank = _world(group)
        self.group, self.backend = group, backend
        self.E, self.k, self.dim, self.hidden = E, k, dim, hidden
        self.e0, self.e1 = expert_range(E, self.rank, self.world)
        self.router = router
        self.mats = []
        for w, t in ((w1, t1), (w3, t3), (w2, t2)):
            w = np.asarray(w, np.uint8)
            local = w[self.e0:self.e1]
            stride = int(np.prod(w.shape[1:])) if w.ndim > 1 else 0
            self.mats.append((backend.upload(local), stride, t))

    def __call__(self, xb, logits=None):
        T = xb.shape[0]
        sel, wts = self.backend.route(xb, self.E, self.k, router=self.router, logits=logits)
        o = self.backend.zeros(T * self.k, self.dim)
        if self.e1 > self.e0:
            self.backend.experts(o, xb, sel, self.e0, self.e1 - self.e0, self.mats, self.dim, self.hidden)
        if self.world > 1:
            dist.all_reduce(o, op=dist.ReduceOp.SUM, group=self.group)
        return self.backend.combine(o, sel, wts, self.dim), sel, wts
