"""Multi-GPU row-slab sharding (one process per GPU, torch.distributed over NCCL).

The reference is single-device; these wrappers partition the pair representation
by pair-row slabs, rank r owning rows [r*N/P, (r+1)*N/P), and use a collective
only where the algorithm exchanges data:

* triangle attention (starting node): rows are independent given the bias
  Bp[h, q, k], which every row shares. Each rank projects its slab (its rows of
  Bp come out of the same GEMM), the Bp slabs are all-gathered, then attention and
  the gate run on local rows. Per rank the exchange is H*N*N*(P-1)/P elements
  (29 MB at N=2048, P=8).
* triangle multiplicative update (x replicated, as in the 1/2/4/8-GPU configuration):
  by channel: the contraction is independent per channel d, so each rank contracts
  C/P channel planes after an input phase over all tokens, and one all-to-all hands
  every rank y of its rows (C*L*L/P^2 elements per peer). By rows (the chain, where x
  is row-sharded): output row i needs a[., i, .] and ALL of b; each rank runs the
  input phase on the token slab that yields its a and its share of b, b's chunks are
  exchanged peer by peer and contracted as they arrive, and the output phase runs on
  the rank's rows.

* attention with pair bias: the bias is per query row, so rank r takes query rows
  [r*M/P, (r+1)*M/P) with its rows of z (the pair tensor, the only large input)
  and the whole single sequence X (M x c_s, a few hundred KB), from which it
  projects K and V for every key itself. No collective: the M*2*H*D K/V elements
  are cheaper to recompute than to exchange.

* the Pairformer chain (``pair_update_rows``): row-sharded x, with all-to-all
  transposes where a step needs columns (incoming multiplication, ending node).

The per-rank compute steps are looked up on an ``ops`` object so that the host
logic (slab partitioning, collective assembly) is testable with gloo on CPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def slab(N: int, rank: int, world: int) -> tuple[int, int]:
    """Row range [r0, r1) of ``rank``; N must divide evenly."""
    if N % world:
        raise AssertionError(f"N={N} is not divisible by world size {world}")
    n = N // world
    return rank * n, (rank + 1) * n


def all_gather_rows(local: torch.Tensor, dim: int, group=None) -> torch.Tensor:
    """All-gather equal slabs along ``dim`` (rank order) into one tensor."""
    world = dist.get_world_size(group)
    if world == 1:
        return local
    moved = local.movedim(dim, 0).contiguous()
    out = torch.empty((world * moved.shape[0],) + moved.shape[1:], dtype=moved.dtype, device=moved.device)
    dist.all_gather_into_tensor(out, moved, group=group)
    return out.movedim(0, dim).contiguous()


class KernelOps:
    """The sm_100a kernels for one rank's slab."""

    @staticmethod
    def project(X_rows, pre, mask_rows, N, scale, eps):
        from .triangle_attn.kernel import project_rows

        w = pre["W_qkvz"] if pre["W_qkvz"].dtype == X_rows.dtype else pre["W_qkvz"].to(X_rows.dtype)
        return project_rows(X_rows, w, pre["ln_w32"], pre["ln_b32"], pre["BZ"], pre["H"], pre["D"], N=N,
                            mask_rows=mask_rows, scale=scale, eps=eps)

    @staticmethod
    def attend(ws, bias_full, pre):
        from .triangle_attn.kernel import attend_rows

        return attend_rows(ws, bias_full, pre["H"], pre["D"])

    @staticmethod
    def gate(O, ws, W_proj_g, W_proj_o):
        from .triangle_attn.kernel import gate_forward

        return gate_forward(O, ws["xln"], W_proj_g, W_proj_o).view(O.shape[0], O.shape[1], -1)


def triangle_attention_rows(X_rows, pre, *, N, mask_rows=None, scale=1.0, eps=1e-5, W_proj_g, W_proj_o, group=None,
                            ops=KernelOps):
    """Starting-node triangle attention of this rank's pair rows X_rows (n, N, C);
    returns the same rows of the output (n, N, C). Collective: all-gather of the
    shared bias slabs (H, n, Np) -> (H, N, Np)."""
    ws = ops.project(X_rows, pre, mask_rows, N, scale, eps)
    bias_full = all_gather_rows(ws["bias"], 1, group)
    O = ops.attend(ws, bias_full, pre)
    return ops.gate(O, ws, W_proj_g, W_proj_o)


class TrimulKernelOps:
    """The sm_100a kernels for one rank's triangle-mul slab."""

    COL_TILE = 256  # contract_cols ranges start on (and span) multiples of this

    @staticmethod
    def contract(a, b, direction):
        from .triangle_mul.kernel import contract

        return contract(a, b, direction)

    @staticmethod
    def contract_cols(a, b_flat, direction, Mi, L, P, j0, jc, y):
        from .triangle_mul.kernel import contract_slab_cols

        contract_slab_cols(a, b_flat, direction, Mi, L, P, j0, jc, y)

    @staticmethod
    def input_phase(x_tokens, mask_tokens, pre, eps):
        from .triangle_mul.kernel import input_phase_tokens

        return input_phase_tokens(x_tokens, mask_tokens, pre, eps)

    @staticmethod
    def contract_slab(a, b_chunks, direction, Mi, L, P):
        from .triangle_mul.kernel import contract_slab

        return contract_slab(a, b_chunks, direction, Mi, L, P)

    @staticmethod
    def output_phase(y, x_tokens, pre, eps):
        from .triangle_mul.kernel import output_phase_tokens

        return output_phase_tokens(y, x_tokens, pre, eps)


def exchange_chunks(chunk, rank, world, group, on_chunk):
    """All-gather of equal chunks (rank-major, as all_gather_into_tensor lays them out)
    that hands each chunk to ``on_chunk(src, flat)`` as soon as it has arrived, the
    caller's own chunk first. Step s of world-1 pairs every rank r with r+s (send) and
    r-s (receive); on CUDA the transfers run on a side stream and each on_chunk call is
    enqueued on the caller's stream behind an event of its transfer, so the work on a
    chunk overlaps the transfers of the later ones. Returns the filled (world, ...) buffer."""
    flat = torch.empty((world,) + tuple(chunk.shape), dtype=chunk.dtype, device=chunk.device)
    flat[rank].copy_(chunk)
    on_chunk(rank, flat)
    cuda = chunk.is_cuda
    if cuda:
        main = torch.cuda.current_stream(chunk.device)
        side = _comm_stream(chunk.device)
        side.wait_stream(main)  # the chunk (and flat) are ready on the caller's stream
        chunk.record_stream(side)
        flat.record_stream(side)
    for step in range(1, world):
        dst, src = (rank + step) % world, (rank - step) % world
        if cuda:
            with torch.cuda.stream(side):
                reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, chunk, dst, group),
                                               dist.P2POp(dist.irecv, flat[src], src, group)])
                for r in reqs:
                    r.wait()
                ev = torch.cuda.Event()
                ev.record(side)
            main.wait_event(ev)
        else:
            for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, chunk, dst, group),
                                             dist.P2POp(dist.irecv, flat[src], src, group)]):
                r.wait()
        on_chunk(src, flat)
    return flat


_COMM = {}


def _comm_stream(device):
    """One side stream per device for the chunked collectives."""
    key = torch.device(device).index
    if key not in _COMM:
        _COMM[key] = torch.cuda.Stream(device=device)
    return _COMM[key]


def _trimul_from_slabs(x_rows, x_cols, pre, direction, mask, eps, group, ops):
    """The triangle multiplicative update of this rank's pair rows from its row slab
    x_rows (n, L, C) = x[r0:r1] and, for the incoming direction, its column slab
    x_cols (L, n, C) = x[:, r0:r1] (any strides; the all-to-all of ``column_blocks``
    delivers it contiguous). mask: the full (L, L) mask or None."""
    n, L, C = x_rows.shape
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    r0, r1 = slab(L, rank, world)
    if direction == "outgoing":  # a rows i in slab, b rows j in slab: tokens (i, k)
        xs = x_rows.reshape(n * L, C)
        ms = None if mask is None else mask.reshape(L, L)[r0:r1].reshape(n * L)
    else:  # a columns i in slab, b columns j in slab: tokens (k, i)
        xs = x_cols.contiguous().reshape(L * n, C)
        ms = None if mask is None else mask.reshape(L, L)[:, r0:r1].contiguous().reshape(L * n)
    ab = ops.input_phase(xs.contiguous(), ms, pre, eps)  # (2C, n*L) as [d][i][k] or [d][k][i]
    a = ab[:C].reshape(C, n, L) if direction == "outgoing" else ab[:C].reshape(C, L, n)
    b = ab[C:].reshape(C, n, L) if direction == "outgoing" else ab[C:].reshape(C, L, n)
    nc = L // world
    tile = getattr(ops, "COL_TILE", None)
    if world > 1 and tile is not None and nc % tile == 0:
        # b's chunks arrive one peer at a time on a side stream; each chunk's output
        # columns are contracted as soon as it lands, the rank's own chunk first
        y = torch.empty(C, n, L, dtype=a.dtype, device=a.device)
        a = a.contiguous()

        def on_chunk(src, flat):
            ops.contract_cols(a, flat, direction, n, L, world, src * nc, nc, y)

        exchange_chunks(b.contiguous(), rank, world, group, on_chunk)
    else:
        if world > 1:
            flat = torch.empty((world * b.shape[0],) + tuple(b.shape[1:]), dtype=b.dtype, device=b.device)
            dist.all_gather_into_tensor(flat, b.contiguous(), group=group)  # rank-major concatenation
            b_chunks = flat.view((world,) + tuple(b.shape))
        else:
            b_chunks = b.unsqueeze(0)
        y = ops.contract_slab(a, b_chunks, direction, n, L, world)  # (C, n, L)
    out = ops.output_phase(y.reshape(C, n * L), x_rows.reshape(n * L, C).contiguous(), pre, eps)
    return out.reshape(n, L, C)


def triangle_multiplicative_update_rows(x, pre, *, direction, mask=None, eps=1e-5, group=None, ops=TrimulKernelOps,
                                        split="auto"):
    """Rows [r0, r1) of the triangle multiplicative update of the replicated pair tensor
    x (1, L, L, C); returns (1, n, L, C).

    split="channels" (the default when C divides by the world size): every rank runs the
    input phase on all tokens, contracts only its C/P channel planes (the contraction is
    independent per channel) and one all-to-all brings each rank y of its rows, all
    channels (C*L*L/P^2 elements to every peer). split="rows": the input phase on the
    rank's share of tokens and b exchanged peer by peer under the row-slab contraction
    (C*L*L*(P-1)/P elements per rank)."""
    if direction not in ("outgoing", "incoming"):
        raise ValueError(f"unknown direction: {direction!r} (expected 'outgoing'/'incoming')")
    B, L, _, C = x.shape
    assert B == 1, "row-slab sharding takes one pair tensor"
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    r0, r1 = slab(L, rank, world)
    if split not in ("auto", "channels", "rows"):
        raise ValueError(f"unknown split: {split!r}")
    if world > 1 and split != "rows" and C % world == 0 and hasattr(ops, "contract"):
        return _trimul_channels(x, pre, direction, mask, eps, group, ops, rank, world)
    x_cols = None if direction == "outgoing" else x[0, :, r0:r1]
    return _trimul_from_slabs(x[0, r0:r1], x_cols, pre, direction, mask, eps, group, ops).unsqueeze(0)


def _trimul_channels(x, pre, direction, mask, eps, group, ops, rank, world):
    """Channel-sharded triangle multiplication of the replicated x (1, L, L, C)."""
    _, L, _, C = x.shape
    n, cs = L // world, C // world
    r0, r1 = rank * n, (rank + 1) * n
    xs = x[0].reshape(L * L, C).contiguous()
    ms = None if mask is None else mask.reshape(L * L)
    ab = ops.input_phase(xs, ms, pre, eps)  # (2C, L*L) D-major: a = channels [0, C), b = [C, 2C)
    d0 = rank * cs
    a = ab[d0:d0 + cs].view(cs, 1, L, L)
    b = ab[C + d0:C + d0 + cs].view(cs, 1, L, L)
    y_mine = ops.contract(a, b, direction)  # this rank's channels of y, every row i
    send = y_mine.reshape(cs, world, n, L).permute(1, 0, 2, 3).contiguous()  # [dest rank][d][i][j]
    recv = torch.empty_like(send)  # [src rank][d of src][i of mine][j]: y of my rows, channel-major
    dist.all_to_all_single(recv.view(-1), send.view(-1), group=group)
    out = ops.output_phase(recv.view(C, n * L), x[0, r0:r1].reshape(n * L, C).contiguous(), pre, eps)
    return out.reshape(1, n, L, C)


def column_blocks(x_rows, group=None):
    """Rows [r0, r1) of x (n, N, C) -> this rank's columns x[:, r0:r1] as a contiguous
    (world, n, n, C) = [src][i of src's rows][k of my columns][C], i.e. (N, n, C), by one
    all-to-all: rank r sends its (n, n, C) block of columns [j0, j1) to rank j."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    n, N, C = x_rows.shape
    if world == 1:
        return x_rows.reshape(1, n, N, C)
    assert n * world == N
    send = x_rows.reshape(n, world, n, C).permute(1, 0, 2, 3).contiguous()  # [dest][i][k][C]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv.view(-1), send.view(-1), group=group)
    return recv


def transpose_rows(x_rows, group=None):
    """Rows [r0, r1) of x (n, N, C) -> the same rows of x^T, i.e. x[:, r0:r1]^T (n, N, C)."""
    n, N, C = x_rows.shape
    return column_blocks(x_rows, group).permute(2, 0, 1, 3).reshape(n, N, C)  # x^T[k][src * n + i]


def pair_update_rows(x_rows, pre, *, mask=None, scale=None, eps=1e-5, group=None, attn_ops=KernelOps,
                     trimul_ops=TrimulKernelOps):
    """The Pairformer pair-update chain (``pairformer.pair_update``) on a row-sharded pair
    tensor: x_rows (n, N, C) holds rows [r0, r1) of x, mask is the full (N, N) mask (or
    None) on every rank; returns the updated rows. Collectives: the b all-gathers of the
    two triangle multiplications, the shared-bias all-gathers of the two attentions, and
    three all-to-all transposes (x^T for the incoming multiplication and the ending-node
    attention, and the ending node's result back to rows)."""
    n, N, _ = x_rows.shape
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    r0, r1 = slab(N, rank, world)
    m = None if mask is None else mask.reshape(N, N)
    x_rows = x_rows + _trimul_from_slabs(x_rows, None, pre["tri_mul_out"], "outgoing", m, eps, group, trimul_ops)
    # the all-to-all delivers x[:, r0:r1] in exactly the token order the incoming input
    # phase reads: no transpose copy on either side of it
    x_cols = column_blocks(x_rows, group).view(N, n, -1)
    x_rows = x_rows + _trimul_from_slabs(x_rows, x_cols, pre["tri_mul_in"], "incoming", m, eps, group, trimul_ops)
    del x_cols
    for name, ending in (("tri_attn_start", False), ("tri_attn_end", True)):
        p = pre[name]
        sc = p["D"] ** -0.5 if scale is None else scale
        src = transpose_rows(x_rows, group) if ending else x_rows
        mr = None if m is None else (m.t() if ending else m)[r0:r1].contiguous()
        o = triangle_attention_rows(src.contiguous(), p, N=N, mask_rows=mr, scale=sc, eps=eps,
                                    W_proj_g=p["W_proj_g"], W_proj_o=p["W_proj_o"], group=group, ops=attn_ops)
        if ending:
            # x[i][src*n + k] += o^T: added through a permuted view of the received blocks,
            # in place (x_rows is this function's own tensor by now), without a transpose copy
            blk = column_blocks(o, group)  # [src][k of src's rows][i of mine][C]
            x_rows.view(n, world, n, -1).add_(blk.permute(2, 0, 1, 3))
        else:
            x_rows = x_rows + o
    return x_rows


class ApbKernelOps:
    """The sm_100a kernels for one rank's query rows of attention with pair bias."""

    @staticmethod
    def attend_rows(X, Z_rows, pre, q0, scale, eps, key_mask):
        from .attn_pair_bias.kernel import apb_core

        H, D = pre["H"], pre["D"]
        w = pre["w_rows"] if pre["w_rows"].dtype == X.dtype else pre["w_rows"].to(X.dtype)
        Og = torch.empty(Z_rows.shape[0], H * D, device=X.device, dtype=X.dtype)
        return apb_core(X, w, Z_rows, pre["W_combined"], pre["sum_W_combined"], pre["B_const"], Og, H, D,
                        scale=scale, eps=eps, key_mask=key_mask, q0=q0)

    @staticmethod
    def gate(Og, X_rows, W_proj_g, B_proj_g, W_proj_o, B_proj_o):
        from .triangle_attn.kernel import gate_forward

        return gate_forward(Og, X_rows, W_proj_g, W_proj_o, B_proj_g, B_proj_o)


def attention_pair_bias_rows(X, Z_rows, pre, *, scale=1.0, eps=1e-5, W_proj_g, B_proj_g, W_proj_o, B_proj_o,
                             mask=None, group=None, ops=ApbKernelOps):
    """This rank's query rows of attention with pair bias: X (M, c_s) the whole
    (replicated) single sequence, Z_rows (n, M, C_z) the rank's pair rows
    z[r0:r1]; returns (n, c_s) = rows [r0, r1) of the unsharded output. No collective."""
    M = X.shape[0]
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    r0, r1 = slab(M, rank, world)
    assert Z_rows.shape[:2] == (r1 - r0, M), f"Z_rows must be z[{r0}:{r1}] of shape ({r1 - r0}, {M}, C_z)"
    Og = ops.attend_rows(X, Z_rows, pre, r0, scale, eps, mask)
    return ops.gate(Og, X[r0:r1].contiguous(), W_proj_g, B_proj_g, W_proj_o, B_proj_o)
