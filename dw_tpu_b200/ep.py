"""Expert-parallel MoE on B200: the one-shot NVLink exchange (dwm_ep_*) and
the EP layer built on it.

The reference's GMM_EP path all-gathers every rank's tokens and routing
(``all_gather_local``, KO:152-164), sorts the gathered batch and keeps the rows
of the rank's own experts (X0101:56-104, X0107:34-51), runs the grouped
matmuls, then forms a masked f32 partial combine over all gathered tokens and
reduce-scatters it (X0107:15-29, ``reduce_scatter_local`` KO:167-185). Here a
rank instead stores each of its (token, k) rows straight into the expert
owner's receive buffer, in the same receive order; the owner's grouped matmul
writes into its output buffer, from which the token owner loads each (token,
k) output and forms the k-order combine (KC:14-21). One kernel each way. One
process per GPU; peers' buffers are mapped with CUDA IPC, exchanged once over
``torch.distributed``.

``NcclExchange`` (NCCL ``all_to_all_single``) and ``all_gather_local`` /
``reduce_scatter_local`` (the reference's collectives on
``torch.distributed``) below are the NCCL comparison paths.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops
from .fused_moe import FP4MoEWeights


class _DeviceArray:
    """Zero-copy ``__cuda_array_interface__`` view of library-owned memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape),
                                         "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class EPContext:
    """One rank's side of the exchange (``dwm_ep_create``): its symmetric
    buffer, the receive view and the receive group sizes.

    Rank ``rank`` of ``world`` owns experts [rank*E/world, (rank+1)*E/world).
    ``recv`` is a bf16 [capacity, hidden] view of the receive buffer and
    ``output(dtype)`` a [capacity, hidden] view of the output buffer, where the
    expert outputs should be written (both owned by the context: keep the
    context alive while they are used)."""

    def __init__(self, rank: int, world: int, *, max_tokens: int, hidden: int, topk: int,
                 num_experts: int):
        self.rank, self.world = int(rank), int(world)
        self.max_tokens, self.hidden, self.topk = int(max_tokens), int(hidden), int(topk)
        self.num_experts = int(num_experts)
        self.local_experts = self.num_experts // self.world if self.world else 0
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = L.lib()
        ctx = ctypes.c_void_p()
        L.check(lib.dwm_ep_create(self.rank, self.world, self.max_tokens, self.hidden,
                                  self.topk, self.num_experts, ctypes.byref(ctx)),
                "dwm_ep_create")
        self._ctx = ctx
        recv = ctypes.c_void_p()
        cap = ctypes.c_int64()
        L.check(lib.dwm_ep_recv_buffer(ctx, ctypes.byref(recv), ctypes.byref(cap)),
                "dwm_ep_recv_buffer")
        self.capacity = cap.value
        self.recv = torch.as_tensor(_DeviceArray(recv.value, (self.capacity, self.hidden), "<i2"),
                                    device=self.device).view(torch.bfloat16)
        outb = ctypes.c_void_p()
        L.check(lib.dwm_ep_output_buffer(ctx, ctypes.byref(outb), ctypes.byref(cap)),
                "dwm_ep_output_buffer")
        self._outb = outb.value
        self.recv_group_sizes = torch.zeros(self.local_experts, dtype=torch.int32,
                                            device=self.device)
        self.num_tokens = 0

    def output(self, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """[capacity, hidden] view of the output buffer (bf16 or f32)."""
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("the output buffer holds bf16 or f32")
        typestr = "<i2" if dtype == torch.bfloat16 else "<f4"
        t = torch.as_tensor(_DeviceArray(self._outb, (self.capacity, self.hidden), typestr),
                            device=self.device)
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    # -- wiring -------------------------------------------------------------
    def ipc_handle(self) -> bytes:
        buf = (ctypes.c_char * L.EP_HANDLE_BYTES)()
        L.check(L.lib().dwm_ep_ipc_handle(self._ctx, buf), "dwm_ep_ipc_handle")
        return bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        if len(handles) != self.world or any(len(h) != L.EP_HANDLE_BYTES for h in handles):
            raise ValueError("expected one IPC handle per rank")
        blob = b"".join(handles)
        L.check(L.lib().dwm_ep_connect(self._ctx, blob), "dwm_ep_connect")

    @staticmethod
    def connect_local(ctxs: list["EPContext"]) -> None:
        arr = (ctypes.c_void_p * len(ctxs))(*[c._ctx.value for c in ctxs])
        for c in ctxs:
            L.check(L.lib().dwm_ep_connect_local(c._ctx, arr), "dwm_ep_connect_local")

    # -- exchange -----------------------------------------------------------
    def dispatch(self, hidden: torch.Tensor, topk_ids: torch.Tensor, *, phases: int = L.EP_ALL,
                 stream: int | None = None):
        """hidden bf16 [T, H], topk_ids int32 [T, topk] -> (recv view
        [capacity, H], recv_group_sizes int32 [E/world]); rows
        [0, sum(recv_group_sizes)) are valid."""
        L.require_cuda(hidden, topk_ids)
        if hidden.dtype != torch.bfloat16 or topk_ids.dtype != torch.int32:
            raise ValueError("hidden must be bf16 and topk_ids int32")
        t = hidden.shape[0]
        if hidden.shape != (t, self.hidden) or topk_ids.shape != (t, self.topk):
            raise ValueError(f"expected hidden [T, {self.hidden}] and ids [T, {self.topk}]")
        hidden, topk_ids = hidden.contiguous(), topk_ids.contiguous()
        self.num_tokens = t
        L.check(L.lib().dwm_ep_dispatch(self._ctx, hidden.data_ptr(), topk_ids.data_ptr(), t,
                                        self.recv_group_sizes.data_ptr(), phases,
                                        L.stream_ptr() if stream is None else stream),
                "dwm_ep_dispatch")
        return self.recv, self.recv_group_sizes

    def combine(self, y: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None, *, phases: int = L.EP_PUSH | L.EP_REDUCE,
                stream: int | None = None, shared: torch.Tensor | None = None,
                routed_scale: float = 1.0, f32_reduce: bool = False,
                rank_order: bool = False) -> torch.Tensor | None:
        """y [rows, H] expert outputs in receive order (bf16 or f32; best the
        ``output()`` view, else they are copied there first), topk_weights
        [T, topk] of this rank's dispatched tokens -> out [T, H] (bf16 unless
        ``out`` says otherwise). ``shared`` [T, H] (bf16/f32): the shared
        expert summed in as ``combine_shared`` does (X0104:80-87).
        ``rank_order``: the reference GMM_EP sum order (per-rank masked f32
        partials, summed over ranks in rank order; X0107:15-29, KO:181-184)
        instead of the k order."""
        if rank_order:
            phases |= L.EP_RANK_ORDER
        L.require_cuda(y, topk_weights)
        if y.dim() != 2 or y.shape[1] != self.hidden or not y.is_contiguous():
            raise ValueError(f"y must be a contiguous [rows, {self.hidden}] tensor")
        t = self.num_tokens
        if topk_weights.shape != (t, self.topk):
            raise ValueError(f"topk_weights must be [{t}, {self.topk}]")
        if out is None and phases & L.EP_REDUCE:
            out = torch.empty((t, self.hidden), dtype=torch.bfloat16, device=y.device)
        if shared is not None:
            L.require_cuda(shared)
            if shared.shape != (t, self.hidden) or shared.dtype not in (torch.bfloat16,
                                                                       torch.float32):
                raise ValueError(f"shared must be bf16/f32 [{t}, {self.hidden}]")
            shared = shared.contiguous()
        L.check(L.lib().dwm_ep_combine_shared(
            self._ctx, y.data_ptr(), L.dtype_code(y.dtype), topk_weights.contiguous().data_ptr(),
            L.dtype_code(topk_weights.dtype), L.ptr(shared),
            L.dtype_code(shared.dtype) if shared is not None else L.F32, float(routed_scale),
            L.F32 if f32_reduce else L.BF16, L.ptr(out),
            L.dtype_code(out.dtype) if out is not None else L.BF16, phases,
            L.stream_ptr() if stream is None else stream), "dwm_ep_combine_shared")
        return out

    def gmm(self, lhs: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
            out: torch.Tensor | None, *, mode: int, act: int = L.ACT_NONE,
            act_limit: float = 0.0, out_dtype: torch.dtype = torch.bfloat16,
            variant: int = 7, stream: int | None = None) -> None:
        """The grouped matmul of the overlapped exchange (dwm_ep_gmm_fp4) on
        the B200-layout weights of this rank's experts: ``mode`` EP_GEMM_GATED
        reads the receive buffer (lhs = ``recv``) expert by expert as the rows
        arrive and writes ``out``; EP_GEMM_PUSH stores every output row into
        its token owner's buffer (``out`` unused). ``variant`` 1 runs the
        one-CTA tcgen05 kernel, 3 / 4 / 5 the mma.sync decode kernel with 8 /
        16 / 32-row tiles, 7 the CTA-pair kernel, 9 the CTA-pair kernel with
        tiles of up to 512 rows."""
        L.require_cuda(lhs, codes, scales)
        sc = scales.view(torch.uint8) if scales.element_size() == 1 else scales
        g, n, k2 = codes.shape
        if g != self.local_experts or lhs.shape[1] != 2 * k2:
            raise ValueError("codes must be this rank's experts in the B200 layout "
                             "[E/world, n, k/2] matching lhs")
        k = 2 * k2
        if sc.numel() != g * (k // 32) * n or not sc.is_contiguous() or not codes.is_contiguous():
            raise ValueError(f"scales must be contiguous [{g}, {k // 32}, {n}] and codes "
                             "contiguous")
        if mode == L.EP_GEMM_GATED:
            n_out = n if act == L.ACT_NONE else n // 2
            if out is None or out.shape != (self.capacity, n_out) or not out.is_contiguous():
                raise ValueError(f"the gated matmul writes a contiguous out "
                                 f"[{self.capacity}, {n_out}]")
            if lhs.data_ptr() != self.recv.data_ptr():
                raise ValueError("the gated matmul reads the receive buffer (lhs = recv)")
        elif mode == L.EP_GEMM_PUSH:
            if act != L.ACT_NONE or n != self.hidden or lhs.shape[0] != self.capacity:
                raise ValueError("the pushing matmul is the down projection: no activation, "
                                 f"n = {self.hidden}, lhs [{self.capacity}, k]")
        else:
            raise ValueError(f"unknown mode {mode}")
        odt = out.dtype if out is not None else out_dtype
        L.check(L.lib().dwm_ep_gmm_fp4(
            self._ctx, lhs.data_ptr(), codes.view(torch.uint8).data_ptr(), L.FP4_B200,
            sc.data_ptr(), L.dtype_code(sc.dtype), self.recv_group_sizes.data_ptr(), 2 * k2, n,
            int(act), float(act_limit), L.dtype_code(odt), L.ptr(out), int(mode), int(variant),
            L.stream_ptr() if stream is None else stream), "dwm_ep_gmm_fp4")

    def link_probe(self, peer: int, nbytes: int, stream: int | None = None) -> None:
        """Copy nbytes of this rank's receive buffer into ``peer``'s over
        NVLink (dwm_ep_link_probe); only between steps, every rank idle."""
        L.check(L.lib().dwm_ep_link_probe(self._ctx, int(peer), int(nbytes),
                                          L.stream_ptr() if stream is None else stream),
                "dwm_ep_link_probe")

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of every device-side wait of later launches (default 2 s). A
        wait that runs out reports DWM_DEV_TIMEOUT (``_lib.DeviceError`` on the
        next status check); every rank's context must then be re-created."""
        L.check(L.lib().dwm_ep_set_wait_limit(self._ctx, int(seconds * 1e9)),
                "dwm_ep_set_wait_limit")

    def close(self) -> None:
        if getattr(self, "_ctx", None) is not None and self._ctx.value:
            L.lib().dwm_ep_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All-gather one fixed-size handle per rank, in rank order."""
    if len(handle) != L.EP_HANDLE_BYTES:
        raise ValueError(f"handle must be {L.EP_HANDLE_BYTES} bytes")
    world = dist.get_world_size(group)
    handles: list = [None] * world
    dist.all_gather_object(handles, bytes(handle), group=group)
    if any(not isinstance(h, bytes) or len(h) != L.EP_HANDLE_BYTES for h in handles):
        raise RuntimeError("a rank sent a malformed IPC handle")
    return handles


def create_context(group=None, *, max_tokens: int, hidden: int, topk: int,
                   num_experts: int) -> EPContext:
    """Collective: every rank of ``group`` creates its context on its current
    device, the IPC handles are all-gathered, and every rank maps its peers."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    ctx = EPContext(rank, world, max_tokens=max_tokens, hidden=hidden, topk=topk,
                    num_experts=num_experts)
    ctx.connect(exchange_handles(ctx.ipc_handle(), group))
    dist.barrier(group=group)
    return ctx


def create_local_contexts(world: int, **kw) -> list[EPContext]:
    """All ``world`` ranks' contexts in this process on the current device:
    the exchange emulated on one GPU (drive it with ``emulated_dispatch`` and
    ``emulated_combine``, which issue every rank's phases in order)."""
    ctxs = [EPContext(r, world, **kw) for r in range(world)]
    EPContext.connect_local(ctxs)
    return ctxs


def emulated_dispatch(ctxs: list[EPContext], hiddens, ids):
    for phase in (L.EP_COUNTS, L.EP_ROWS, L.EP_WAIT):
        for c, h, i in zip(ctxs, hiddens, ids):
            c.dispatch(h, i, phases=phase)
    return [(c.recv, c.recv_group_sizes) for c in ctxs]


def emulated_combine(ctxs: list[EPContext], ys, weights, outs=None, rank_order: bool = False):
    outs = outs or [None] * len(ctxs)
    for c, y, w in zip(ctxs, ys, weights):
        c.combine(y, w, None, phases=L.EP_PUSH)
    return [c.combine(y, w, o, phases=L.EP_REDUCE, rank_order=rank_order)
            for c, y, w, o in zip(ctxs, ys, weights, outs)]


# ---------------------------------------------------------------------------
# NCCL comparison path: the reference's collectives
# ---------------------------------------------------------------------------

class NcclExchange:
    """The NCCL comparison path of the EP exchange: ``all_to_all_single`` of
    per-expert counts, then of the token rows themselves (sorted by expert on
    the sender), a local reorder into the one-shot path's receive order
    (expert-major, then source rank, source token, k slot), and on the way back
    an ``all_to_all_single`` of the expert outputs followed by the same k-order
    combine (KC:44-54). Receive buffers and outputs equal the one-shot
    kernels' bit for bit; the price is NCCL's uneven splits, which need the
    counts on the host (one device-to-host sync per dispatch)."""

    def __init__(self, num_experts: int, hidden: int, topk: int, group=None):
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if num_experts % self.world:
            raise ValueError("num_experts must divide by the world size")
        self.num_experts, self.hidden, self.topk = int(num_experts), int(hidden), int(topk)
        self.local_experts = self.num_experts // self.world

    def dispatch(self, hidden: torch.Tensor, topk_ids: torch.Tensor):
        """hidden [T, H], topk_ids int32 [T, topk] (every id in range) ->
        (received rows [R, H] in receive order, group sizes int32 [E/world])."""
        t, k, le, world = hidden.shape[0], self.topk, self.local_experts, self.world
        if topk_ids.shape != (t, k) or hidden.shape[1] != self.hidden:
            raise ValueError("expected hidden [T, H] and topk_ids [T, topk]")
        dev = hidden.device
        flat = topk_ids.reshape(-1).long()
        order = torch.argsort(flat, stable=True)  # (expert, token, k) order = by owner rank
        send = hidden.index_select(0, order // k)
        exp_counts = torch.bincount(flat, minlength=self.num_experts).to(torch.int64)
        recv_exp = torch.empty_like(exp_counts)
        dist.all_to_all_single(recv_exp, exp_counts, group=self.group)
        recv_exp = recv_exp.view(world, le)              # [source rank, local expert]
        counts = torch.stack([exp_counts.view(world, le).sum(1), recv_exp.sum(1)]).cpu()
        in_splits, out_splits = counts[0].tolist(), counts[1].tolist()
        recv = torch.empty((sum(out_splits), self.hidden), dtype=hidden.dtype, device=dev)
        dist.all_to_all_single(recv, send, out_splits, in_splits, group=self.group)
        # Row (source s, local expert x, j-th of that block) goes to
        # ebase[x] + (rows of x from sources before s) + j.
        gs = recv_exp.sum(0)
        ebase = torch.cumsum(gs, 0) - gs
        before = torch.cumsum(recv_exp, 0) - recv_exp
        blocks = recv_exp.reshape(-1)
        block_start = torch.cumsum(blocks, 0) - blocks
        n = int(sum(out_splits))
        block_of_row = torch.repeat_interleave(torch.arange(world * le, device=dev), blocks,
                                               output_size=n)
        j = torch.arange(n, device=dev) - block_start[block_of_row]
        x_of_row = block_of_row % le
        dest = ebase[x_of_row] + before.reshape(-1)[block_of_row] + j
        out = torch.empty_like(recv)
        out.index_copy_(0, dest, recv)
        self._state = (order, dest, in_splits, out_splits, t)
        return out, gs.to(torch.int32)

    def return_rows(self, y: torch.Tensor) -> torch.Tensor:
        """Expert outputs y [R, H] in receive order -> each of this rank's
        (token, k) pairs' output row, [T * topk, H] in (token, k) order."""
        order, dest, in_splits, out_splits, t = self._state
        back = torch.empty((t * self.topk, y.shape[1]), dtype=y.dtype, device=y.device)
        dist.all_to_all_single(back, y.index_select(0, dest), in_splits, out_splits,
                               group=self.group)
        rows = torch.empty_like(back)
        rows.index_copy_(0, order, back)
        return rows

    def combine(self, y: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """The k-order combine of this rank's tokens from the expert outputs y
        [R, H] (receive order) and topk_weights [T, topk]."""
        rows = self.return_rows(y)
        t = topk_weights.shape[0]
        if out is None:
            out = torch.empty((t, y.shape[1]), dtype=torch.bfloat16, device=y.device)
        ident = torch.arange(t * self.topk, dtype=torch.int32, device=y.device)
        return ops.combine_out(rows, ident, topk_weights.contiguous(), self.topk, out)


def all_gather_local(x: torch.Tensor, group=None) -> torch.Tensor:
    """KO:152-164: rank-major concatenation of every rank's block (NCCL)."""
    world = dist.get_world_size(group)
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                      device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def reduce_scatter_local(x: torch.Tensor, group=None,
                         out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """KO:167-185: rank r receives the f32 sum over ranks of block r (NCCL's
    summation order, not the reference's rank order)."""
    world = dist.get_world_size(group)
    xf = x.float().contiguous()
    out = torch.empty((x.shape[0] // world,) + tuple(x.shape[1:]), dtype=torch.float32,
                      device=x.device)
    dist.reduce_scatter_tensor(out, xf, op=dist.ReduceOp.SUM, group=group)
    return out.to(out_dtype or x.dtype)


# ---------------------------------------------------------------------------
# The EP layer
# ---------------------------------------------------------------------------

def overlap_variant(expected_rows: float) -> int:
    """Kernel of the overlapped exchange (one that carries its hooks) for a
    local expert receiving ``expected_rows`` rows on average."""
    if expected_rows >= 224:
        return 9  # tcgen05 on CTA pairs, tiles of up to 512 rows
    if expected_rows >= 96:
        return 7  # tcgen05 on CTA pairs
    if expected_rows > 32:
        return 1  # tcgen05, one CTA
    if expected_rows > 16:
        return 5  # mma.sync decode kernel, 32-row tiles
    return 4 if expected_rows > 6 else 3  # mma.sync decode kernel, 16 / 8-row tiles


def gemm_variant(layout: str, expected_rows: float) -> int:
    """Kernel choice for a local expert receiving ``expected_rows`` rows on
    average (the receive buffer's row count is a capacity, not a size)."""
    if layout != "b200":
        return 0
    if expected_rows <= 6:
        return 3  # mma.sync kernel, 8-row token tiles
    if expected_rows <= 16:
        return 4  # mma.sync kernel, 16-row token tiles (one task per expert)
    if expected_rows <= 48:
        return 10  # each group on the kernel for its size (decode kernel up to 32 rows)
    if expected_rows >= 224:
        return 9  # tcgen05 on CTA pairs, tiles of up to 512 rows
    if expected_rows >= 96:
        return 7  # tcgen05 on CTA pairs, tiles of up to 256 rows
    return 1      # tcgen05 kernel, one CTA


class EPMoELayer:
    """Expert-parallel FP4 MoE layer: local routing, one-shot dispatch, the
    two grouped matmuls on the rank's experts, one-shot combine (the GMM_EP
    layer of X0104:88-98 / X0107 with the exchange above).

    ``weights`` holds the rank's E/world experts (global experts
    [rank*E/world, (rank+1)*E/world)); routing runs over all E experts."""

    def __init__(self, weights: FP4MoEWeights, ctx: EPContext, top_k: int, *,
                 scoring_fn: str = "sigmoid", renormalize: bool = True,
                 act_limit: float | None = None, f32_reduce: bool = False,
                 expected_rows: float | None = None, overlap: bool = False,
                 gemm_variant: int | None = None, rank_order: bool = False):
        if weights.num_experts != ctx.local_experts:
            raise ValueError(f"weights hold {weights.num_experts} experts, the context "
                             f"{ctx.local_experts} per rank")
        if top_k != ctx.topk:
            raise ValueError("top_k differs from the context's")
        self.w, self.ctx = weights, ctx
        self.top_k = int(top_k)
        self.scoring_fn, self.renormalize = scoring_fn, renormalize
        self.act = L.ACT_SWIGLU if act_limit is None else L.ACT_SWIGLU_CLAMP
        self.act_limit = 0.0 if act_limit is None else float(act_limit)
        dev = ctx.device
        t, k = ctx.max_tokens, self.top_k
        self.ids = torch.empty((t, k), dtype=torch.int32, device=dev)
        self.w16 = torch.empty((t, k), dtype=torch.bfloat16, device=dev)
        cap, i, h = ctx.capacity, weights.intermediate_size, weights.hidden_size
        self.h1 = torch.empty((cap, i), dtype=torch.bfloat16, device=dev)
        self.y = ctx.output(torch.float32 if f32_reduce else torch.bfloat16)
        if expected_rows is None:  # uniform routing over all experts
            expected_rows = t * k / ctx.num_experts * ctx.world
        self.variant = (globals()["gemm_variant"](weights.layout, expected_rows)
                        if gemm_variant is None else int(gemm_variant))
        # overlap: the exchange folded into the CTA-pair grouped matmuls
        # (dwm_ep_gmm_fp4): gmm1 starts on each expert as its rows arrive,
        # gmm2 stores its rows straight into the token owners' buffers.
        self.overlap = bool(overlap)
        if self.overlap and weights.layout != "b200":
            raise ValueError("the overlapped exchange takes B200-layout weights")
        if self.overlap:  # the kernels that carry the exchange hooks
            if gemm_variant is None:
                self.variant = overlap_variant(expected_rows)
            elif int(gemm_variant) not in (1, 3, 4, 5, 7, 9):
                raise ValueError("the overlapped exchange runs on variant 1, 3, 4, 5, 7 or 9")
        self.y_dtype = torch.float32 if f32_reduce else torch.bfloat16
        # rank_order: the combine sums in the reference GMM_EP order (per-rank
        # masked f32 partials, then ranks in order) instead of k order.
        self.rank_order = bool(rank_order)
        if self.rank_order and self.overlap:
            raise ValueError("the rank-order combine pulls the peers' rows; the overlapped "
                             "exchange pushes them")

    kernels_per_forward = 5  # route, dispatch, 2 gmm, combine

    def _route(self, logits: torch.Tensor):
        t = logits.shape[0]
        ids, w16 = self.ids[:t], self.w16[:t]
        ops.route_topk_out(logits, self.top_k, ids, w16_out=w16, scoring_fn=self.scoring_fn,
                           renormalize=self.renormalize)
        return ids, w16

    def _experts(self) -> None:
        gs = self.ctx.recv_group_sizes
        ops.gmm_fp4_out(self.ctx.recv, self.w.w13, self.w.s13, gs, self.h1, act=self.act,
                        act_limit=self.act_limit, layout=self.w.layout, variant=self.variant)
        ops.gmm_fp4_out(self.h1, self.w.w2, self.w.s2, gs, self.y, layout=self.w.layout,
                        variant=self.variant)

    def _experts_overlapped(self) -> None:
        c = self.ctx
        c.gmm(c.recv, self.w.w13, self.w.s13, self.h1, mode=L.EP_GEMM_GATED, act=self.act,
              act_limit=self.act_limit, variant=self.variant)
        c.gmm(self.h1, self.w.w2, self.w.s2, None, mode=L.EP_GEMM_PUSH, out_dtype=self.y_dtype,
              variant=self.variant)

    _DISPATCH_OVERLAP = L.EP_COUNTS | L.EP_ROWS | L.EP_GATED
    _COMBINE_OVERLAP = L.EP_REDUCE | L.EP_PUSHED

    def forward(self, hidden: torch.Tensor, logits: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        ids, w16 = self._route(logits)
        if self.overlap:
            self.ctx.dispatch(hidden, ids, phases=self._DISPATCH_OVERLAP)
            self._experts_overlapped()
            return self.ctx.combine(self.y, w16, out, phases=self._COMBINE_OVERLAP)
        self.ctx.dispatch(hidden, ids)
        self._experts()
        return self.ctx.combine(self.y, w16, out, rank_order=self.rank_order)

    __call__ = forward

    @staticmethod
    def forward_emulated(layers: list["EPMoELayer"], hiddens, logits, outs=None):
        """All ranks' layers in one process on one device (contexts from
        ``create_local_contexts``): each exchange phase is issued for every
        rank before the next phase."""
        routed = [ly._route(lg) for ly, lg in zip(layers, logits)]
        if layers[0].overlap:
            outs = outs or [None] * len(layers)
            for phase in (L.EP_COUNTS | L.EP_GATED, L.EP_ROWS | L.EP_GATED):
                for ly, h, (ids, _) in zip(layers, hiddens, routed):
                    ly.ctx.dispatch(h, ids, phases=phase)
            for gated in (True, False):  # every rank's gmm1, then every rank's gmm2
                for ly in layers:
                    c = ly.ctx
                    if gated:
                        c.gmm(c.recv, ly.w.w13, ly.w.s13, ly.h1, mode=L.EP_GEMM_GATED,
                              act=ly.act, act_limit=ly.act_limit, variant=ly.variant)
                    else:
                        c.gmm(ly.h1, ly.w.w2, ly.w.s2, None, mode=L.EP_GEMM_PUSH,
                              out_dtype=ly.y_dtype, variant=ly.variant)
            return [ly.ctx.combine(ly.y, r[1], o, phases=EPMoELayer._COMBINE_OVERLAP)
                    for ly, r, o in zip(layers, routed, outs)]
        emulated_dispatch([ly.ctx for ly in layers], hiddens, [r[0] for r in routed])
        for ly in layers:
            ly._experts()
        return emulated_combine([ly.ctx for ly in layers], [ly.y for ly in layers],
                                [r[1] for r in routed], outs, rank_order=layers[0].rank_order)
