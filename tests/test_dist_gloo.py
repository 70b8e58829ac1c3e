"""World-size-2 gloo test (CPU) of the row-slab sharding host logic: slab
partitioning and the all-gather of the shared triangle-attention bias. The
per-rank kernels are replaced by fp32 torch stand-ins; the result must equal
the unsharded oracle."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import oracle
from triangleops_b200 import dist as tdist


class CpuOps:
    @staticmethod
    def project(X_rows, pre, mask_rows, N, scale, eps):
        n, _, C = X_rows.shape
        H, D = pre["H"], pre["D"]
        xln = F.layer_norm(X_rows, (C,), pre["W_ln"], pre["B_ln"], eps)
        heads = lambda W: (xln @ W).view(n, N, H, D).permute(0, 2, 1, 3)  # noqa: E731
        m = torch.ones(n, N, dtype=torch.bool) if mask_rows is None else mask_rows.bool()
        bias = (xln @ pre["Wz"] + pre["BZ"]).permute(2, 0, 1).contiguous()  # (H, n, N)
        return dict(q=heads(pre["WQ"]) * scale, k=heads(pre["WK"]), v=heads(pre["WV"]), m=m, bias=bias, xln=xln)

    @staticmethod
    def attend(ws, bias_full, pre):
        s = ws["q"] @ ws["k"].transpose(-1, -2) + bias_full[None]
        s = s + torch.where(ws["m"][:, None, None, :], 0.0, -1e9)
        o = torch.softmax(s, -1) @ ws["v"]
        n, H, N, D = o.shape
        return o.permute(0, 2, 1, 3).reshape(n, N, H * D)

    @staticmethod
    def gate(O, ws, Wg, Wo):
        return F.linear(O * torch.sigmoid(F.linear(ws["xln"], Wg)), Wo)


def _inputs():
    g = torch.Generator().manual_seed(7)
    N, H, D, C = 12, 2, 8, 16
    r = lambda *s, sd=1.0: torch.randn(*s, generator=g) * sd  # noqa: E731
    a = dict(X=r(N, N, C), W_ln=1 + 0.1 * r(C), B_ln=0.1 * r(C), WQ=r(C, H * D, sd=C**-0.5),
             WK=r(C, H * D, sd=C**-0.5), WV=r(C, H * D, sd=C**-0.5), Wz=r(C, H, sd=C**-0.5), BZ=0.1 * r(H),
             Wg=r(C, C, sd=C**-0.5), Wo=r(C, C, sd=C**-0.5))
    mask = torch.rand(N, N, generator=g) > 0.2
    return N, H, D, a, mask


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, H, D, a, mask = _inputs()
        r0, r1 = tdist.slab(N, rank, world)
        pre = dict(H=H, D=D, W_ln=a["W_ln"], B_ln=a["B_ln"], WQ=a["WQ"], WK=a["WK"], WV=a["WV"], Wz=a["Wz"],
                   BZ=a["BZ"], W_qkvz=torch.cat([a["WQ"].t(), a["WK"].t(), a["WV"].t()]))
        out = tdist.triangle_attention_rows(a["X"][r0:r1], pre, N=N, mask_rows=mask[r0:r1], scale=D**-0.5,
                                            W_proj_g=a["Wg"], W_proj_o=a["Wo"], ops=CpuOps)
        full = tdist.all_gather_rows(out.contiguous(), 0)
        if rank == 0:
            q.put(full)
        # every rank done before any tears down (gloo teardown races otherwise)
        dist.barrier()
    finally:
        dist.destroy_process_group()


class CpuTrimulOps:
    """fp32 torch stand-ins for the triangle-mul kernels (same layouts)."""

    @staticmethod
    def input_phase(xt, mt, pre, eps):
        w = pre["w"]
        C = xt.shape[1]
        xln = F.layer_norm(xt, (C,), w["norm_in_weight"], w["norm_in_bias"], eps)
        g = F.linear(xln, w["p_in_weight"]) * F.linear(xln, w["g_in_weight"]).sigmoid()
        if mt is not None:
            g = g * mt.float()[:, None]
        return g.t().contiguous()  # (2C, M)

    @staticmethod
    def contract_slab(a, b_chunks, direction, Mi, L, P):
        if direction == "outgoing":  # a (C, Mi, L); b_chunks (P, C, L/P, L)
            b = b_chunks.permute(1, 0, 2, 3).reshape(a.shape[0], L, L)
            return torch.einsum("dik,djk->dij", a, b)
        b = b_chunks.permute(1, 2, 0, 3).reshape(a.shape[0], L, L)  # (C, k, j)
        return torch.einsum("dki,dkj->dij", a, b)

    COL_TILE = 1  # exercise the chunk-by-chunk exchange on CPU

    @staticmethod
    def contract(a, b, direction):  # (D, B, L, L) planes
        if direction == "outgoing":
            return torch.einsum("dbik,dbjk->dbij", a, b)
        return torch.einsum("dbki,dbkj->dbij", a, b)

    @staticmethod
    def contract_cols(a, b_flat, direction, Mi, L, P, j0, jc, y):
        C, nc = a.shape[0], L // P
        ch = b_flat[j0 // nc]  # one chunk: (C, nc, L) outgoing / (C, L, nc) incoming
        if direction == "outgoing":
            y[:, :, j0:j0 + jc] = torch.einsum("dik,djk->dij", a, ch)
        else:
            y[:, :, j0:j0 + jc] = torch.einsum("dki,dkj->dij", a, ch)

    @staticmethod
    def output_phase(y, xt, pre, eps):
        w = pre["w"]
        C = xt.shape[1]
        yt = y.t()
        yln = F.layer_norm(yt, (C,), w["norm_out_weight"], w["norm_out_bias"], eps)
        xln = F.layer_norm(xt, (C,), w["norm_in_weight"], w["norm_in_bias"], eps)
        return F.linear(yln, w["p_out_weight"]) * F.linear(xln, w["g_out_weight"]).sigmoid()


def _trimul_inputs(L=12):
    g = torch.Generator().manual_seed(11)
    C = 16
    r = lambda *s, sd=1.0: torch.randn(*s, generator=g) * sd  # noqa: E731
    w = dict(norm_in_weight=1 + 0.1 * r(C), norm_in_bias=0.1 * r(C), p_in_weight=r(2 * C, C, sd=C**-0.5),
             g_in_weight=r(2 * C, C, sd=C**-0.5), norm_out_weight=1 + 0.1 * r(C), norm_out_bias=0.1 * r(C),
             p_out_weight=r(C, C, sd=C**-0.5), g_out_weight=r(C, C, sd=C**-0.5))
    return r(1, L, L, C), (torch.rand(1, L, L, generator=g) > 0.2), w


def _trimul_worker(rank, world, port, q, direction, split):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, mask, w = _trimul_inputs()
        out = tdist.triangle_multiplicative_update_rows(x, {"w": w}, direction=direction, mask=mask, ops=CpuTrimulOps,
                                                        split=split)
        full = tdist.all_gather_rows(out[0].contiguous(), 0)
        if rank == 0:
            q.put(full)
        # every rank done before any tears down (gloo teardown races otherwise)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split,world", [("rows", 2), ("rows", 3), ("channels", 2), ("channels", 4)])
@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_sharded_triangle_mul_gloo(direction, world, split):
    """Row slabs with b exchanged chunk by chunk (each peer's chunk contracted as it
    arrives; 3 ranks pair every rank with two different peers), and channel planes with
    one all-to-all of y."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_trimul_worker, args=(r, world, port, q, direction, split)) for r in range(world)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, mask, w = _trimul_inputs()
    ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, **w)
    assert (full - ref[0]).abs().max().item() < 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_partition():
    assert tdist.slab(2048, 3, 8) == (768, 1024)
    with pytest.raises(AssertionError):
        tdist.slab(130, 0, 8)


def test_sharded_triangle_attention_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    N, H, D, a, mask = _inputs()
    ref = oracle.triangle_attention(a["X"], a["W_ln"], a["B_ln"], a["WQ"], a["WK"], a["WV"], a["Wz"], a["BZ"],
                                    a["Wg"], None, a["Wo"], None, H, D, scale=D**-0.5, mask=mask)
    assert (full - ref).abs().max().item() < 1e-4


class CpuApbOps:
    """fp32 torch stand-ins for the pair-bias attention kernels (query rows q0..)."""

    @staticmethod
    def attend_rows(X, Z_rows, pre, q0, scale, eps, key_mask):
        w = pre["w"]
        H, D = pre["H"], pre["D"]
        M, n = X.shape[0], Z_rows.shape[0]
        q = (X[q0:q0 + n] @ w["WQ"]).view(n, H, D).transpose(0, 1)
        k = (X @ w["WK"]).view(M, H, D).transpose(0, 1)
        v = (X @ w["WV"]).view(M, H, D).transpose(0, 1)
        bias = (F.layer_norm(Z_rows, Z_rows.shape[-1:], w["W_ln"], w["B_ln"], eps) @ w["Wz"]).permute(2, 0, 1)
        s = q @ k.transpose(-1, -2) * scale + bias
        if key_mask is not None:
            s = s.masked_fill(~key_mask.bool()[None, None, :], float("-inf"))
        return (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(n, H * D)

    @staticmethod
    def gate(Og, X_rows, Wg, Bg, Wo, Bo):
        return F.linear(Og * torch.sigmoid(F.linear(X_rows, Wg, Bg)), Wo, Bo)


def _apb_inputs():
    g = torch.Generator().manual_seed(13)
    M, H, D, Cz = 10, 2, 8, 16
    C = H * D
    r = lambda *s, sd=1.0: torch.randn(*s, generator=g) * sd  # noqa: E731
    w = dict(WQ=r(C, C, sd=C**-0.5), WK=r(C, C, sd=C**-0.5), WV=r(C, C, sd=C**-0.5), W_ln=1 + 0.1 * r(Cz),
             B_ln=0.1 * r(Cz), Wz=r(Cz, H, sd=Cz**-0.5), Wg=r(C, C, sd=C**-0.5), Bg=0.1 * r(C),
             Wo=r(C, C, sd=C**-0.5), Bo=0.1 * r(C))
    km = torch.ones(M, dtype=torch.bool)
    km[-3:] = False
    return r(M, C), r(M, M, Cz), w, km, H, D


def _apb_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        X, Z, w, km, H, D = _apb_inputs()
        r0, r1 = tdist.slab(X.shape[0], rank, world)
        out = tdist.attention_pair_bias_rows(X, Z[r0:r1], {"w": w, "H": H, "D": D}, scale=0.5, W_proj_g=w["Wg"],
                                             B_proj_g=w["Bg"], W_proj_o=w["Wo"], B_proj_o=w["Bo"], mask=km,
                                             ops=CpuApbOps)
        full = tdist.all_gather_rows(out.contiguous(), 0)
        if rank == 0:
            q.put(full)
        # every rank done before any tears down (gloo teardown races otherwise)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_attention_pair_bias_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_apb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    X, Z, w, km, H, D = _apb_inputs()
    ref = oracle.attention_pair_bias_masked(X, w["WQ"], w["WK"], w["WV"], Z, w["W_ln"], w["B_ln"], w["Wz"], None,
                                            w["Wg"], w["Wo"], H, D, key_mask=km, scale=0.5, B_proj_g=w["Bg"],
                                            B_proj_o=w["Bo"])
    assert (full - ref).abs().max().item() < 1e-4


def _chain_inputs():
    g = torch.Generator().manual_seed(21)
    N, C, H, D = 8, 16, 2, 8
    r = lambda *s, sd=1.0: torch.randn(*s, generator=g) * sd  # noqa: E731

    def tm():
        return dict(norm_in_weight=1 + 0.1 * r(C), norm_in_bias=0.1 * r(C), p_in_weight=r(2 * C, C, sd=C**-0.5),
                    g_in_weight=r(2 * C, C, sd=C**-0.5), norm_out_weight=1 + 0.1 * r(C), norm_out_bias=0.1 * r(C),
                    p_out_weight=r(C, C, sd=C**-0.5), g_out_weight=r(C, C, sd=C**-0.5))

    def ta():
        return dict(W_ln=1 + 0.1 * r(C), B_ln=0.1 * r(C), WQ=r(C, H * D, sd=C**-0.5), WK=r(C, H * D, sd=C**-0.5),
                    WV=r(C, H * D, sd=C**-0.5), W_proj_z=r(C, H, sd=C**-0.5), B_proj_z=0.1 * r(H),
                    W_proj_g=r(C, C, sd=C**-0.5), W_proj_o=r(C, C, sd=C**-0.5), H=H, D=D)

    w = dict(tri_mul_out=tm(), tri_mul_in=tm(), tri_attn_start=ta(), tri_attn_end=ta())
    mask = torch.rand(N, N, generator=g) > 0.2
    return r(N, N, C), w, mask


def _chain_pre(w):
    pre = {k: {"w": w[k]} for k in ("tri_mul_out", "tri_mul_in")}
    for k in ("tri_attn_start", "tri_attn_end"):
        a = w[k]
        pre[k] = dict(H=a["H"], D=a["D"], W_ln=a["W_ln"], B_ln=a["B_ln"], WQ=a["WQ"], WK=a["WK"], WV=a["WV"],
                      Wz=a["W_proj_z"], BZ=a["B_proj_z"], W_qkvz=torch.cat([a["WQ"].t(), a["WK"].t(), a["WV"].t()]),
                      W_proj_g=a["W_proj_g"], W_proj_o=a["W_proj_o"])
    return pre


def _chain_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, w, mask = _chain_inputs()
        N = x.shape[0]
        r0, r1 = tdist.slab(N, rank, world)
        out = tdist.pair_update_rows(x[r0:r1].contiguous(), _chain_pre(w), mask=mask, attn_ops=CpuOps,
                                     trimul_ops=CpuTrimulOps)
        full = tdist.all_gather_rows(out.contiguous(), 0)
        if rank == 0:
            q.put(full)
        # every rank done before any tears down (gloo teardown races otherwise)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_transpose_rows_single_rank():
    x = torch.arange(4 * 4 * 3, dtype=torch.float32).reshape(4, 4, 3)
    assert torch.equal(tdist.transpose_rows(x), x.transpose(0, 1))


def test_sharded_pairformer_chain_gloo():
    """Row-sharded chain (all-to-all transposes for the incoming multiplication and the
    ending node) on 2 gloo ranks with CPU stand-ins equals the unsharded oracle chain."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_chain_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, w, mask = _chain_inputs()
    ref = oracle.pair_update(x, mask=mask, **w)
    assert (full - ref).abs().max().item() < 1e-4


def _blocks_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, C = 6 * world, 3
        x = torch.arange(N * N * C, dtype=torch.float32).reshape(N, N, C)
        r0, r1 = tdist.slab(N, rank, world)
        blk = tdist.column_blocks(x[r0:r1].contiguous())
        ok_cols = torch.equal(blk.reshape(N, r1 - r0, C), x[:, r0:r1])
        ok_t = torch.equal(tdist.transpose_rows(x[r0:r1].contiguous()), x.transpose(0, 1)[r0:r1])
        # the chain's in-place add of an ending-node result o (rows of the transposed
        # problem) through a permuted view of its column blocks
        o = -x.transpose(0, 1).contiguous()
        acc = x[r0:r1].clone()
        n = r1 - r0
        acc.view(n, world, n, C).add_(tdist.column_blocks(o[r0:r1].contiguous()).permute(2, 0, 1, 3))
        ok_add = torch.equal(acc, x[r0:r1] + o.transpose(0, 1)[r0:r1])
        q.put((rank, ok_cols, ok_t, ok_add))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_column_blocks_gloo(world):
    """column_blocks delivers x[:, r0:r1] as (N, n, C) in the receive buffer's own layout,
    transpose_rows the rows of x^T, and the permuted in-place add used for the ending node
    equals adding the transposed result."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_blocks_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok_cols and ok_t and ok_add for _, ok_cols, ok_t, ok_add in res), res
