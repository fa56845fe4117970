"""One decode token through the Qwen3.5 hybrid stack's hot path, on one GPU.

Per full-attention layer: fused append-quantize of the new token's K/V into the
layer's paged INT4 pool, then split-KV INT4 decode attention of the query over
it.  Per Gated-DeltaNet layer: the recurrent gated-delta-rule step on the
layer's fp32 state, in place.  Layer order follows Qwen3.5's ``layer_types``
(every ``full_attention_interval``-th layer is full attention,
transformers models/qwen3_5/configuration_qwen3_5.py).  The projections and MLPs
around these kernels are not part of this path.

``HybridDecodeStack.step`` is the host-facing call: it copies the step's
inputs from pinned host memory, runs the step (a captured CUDA graph of every
kernel launch) and copies the outputs back.  ``step_device`` launches the same
kernels on device-resident inputs.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import cabi
from .compression.paged_kv import PageAllocator, PagedKvState


@dataclass
class HybridShape:
    batch: int = 64
    context: int | list[int] = 4096
    num_layers: int = 24
    full_attention_interval: int = 4
    num_heads: int = 8
    num_kv_heads: int = 2
    head_dim: int = 256
    gdn_heads: int = 16
    gdn_dim: int = 128
    page_size: int = 64

    @property
    def layer_types(self) -> list[str]:
        k = self.full_attention_interval
        return ["full_attention" if (i + 1) % k == 0 else "linear_attention" for i in range(self.num_layers)]

    @property
    def lengths(self) -> list[int]:
        if isinstance(self.context, int):
            return [self.context] * self.batch
        return [int(x) for x in self.context]


@dataclass
class _AttnLayer:
    paged: PagedKvState
    write_pos: torch.Tensor      # int32 [B]: slot the new token is written to
    attend_lens: torch.Tensor    # int32 [B]: tokens attended (includes the new one)
    workspace: torch.Tensor
    q: torch.Tensor = None
    k: torch.Tensor = None
    v: torch.Tensor = None
    gate: torch.Tensor = None    # [B, Hq, D] output gate (with epilogues)
    out: torch.Tensor = None


@dataclass
class _GdnLayer:
    state: torch.Tensor
    conv_state: torch.Tensor = None  # [B, C, 4] with the fused causal conv1d update
    conv_w: torch.Tensor = None
    conv_b: torch.Tensor = None
    qkv: torch.Tensor = None         # [B, C] projection output (fused conv) ...
    q: torch.Tensor = None           # ... or q / k / v after the conv
    k: torch.Tensor = None
    v: torch.Tensor = None
    g: torch.Tensor = None           # fp32 [B, 1, H] decay exponent ...
    beta: torch.Tensor = None        # ... and write strength, precomputed (conv variants), or
    a: torch.Tensor = None           # the raw projections [B, 1, H] the step turns into g and beta
    b: torch.Tensor = None
    A_log: torch.Tensor = None       # [H] layer parameters of that gate arithmetic
    dt_bias: torch.Tensor = None
    z: torch.Tensor = None           # [B, 1, H, Dv] gate of the output norm (with epilogues)
    norm_w: torch.Tensor = None      # [Dv] weight of the output norm
    out: torch.Tensor = None


@dataclass
class StepCounts:
    launches: int
    attn_bytes: int          # algorithmic KV bytes read per step (all attention layers)
    gdn_bytes: int           # state bytes read + written per step (all GDN layers)
    append_bytes: int
    h2d_bytes: int
    d2h_bytes: int
    per_kernel: dict = field(default_factory=dict)


class HybridDecodeStack:
    """Device state of the hybrid stack for ``shape.batch`` sequences.

    ``hold_context=True`` keeps every sequence at its configured context: each
    step quantises the new token into slot ``context`` of its page and attends
    over ``context + 1`` tokens, so repeated steps measure the same workload.
    With ``hold_context=False`` the caches grow by one token per step.
    ``conv`` feeds every GDN layer its raw q/k/v projection output and runs the layer's
    causal conv1d update (kernel 4) as the decode branch of Qwen3_5GatedDeltaNet does:
    ``"separate"`` launches ``oq_causal_conv1d_update`` then the GDN step on its output,
    ``"fused"`` the single-launch ``oq_gdn_conv_step`` (slower on B200, measured: the four
    column-slice CTAs of a head each convolve q/k and synchronise as a cluster).  With
    ``conv=None`` q/k/v are given post-conv.
    ``gates="given"`` feeds every GDN step its g and beta, the hook's own arguments;
    ``gates="fused"`` (no conv mode) gives it the raw gate projections ``a``, ``b`` instead and
    computes ``g = -exp(A_log) softplus(a + dt_bias)``, ``beta = sigmoid(b)`` inside the step
    kernel (``oq_gdn_recurrent_gates``), as the decode branch does ahead of the hook.
    ``epilogues=True`` adds the layers' output epilogues: the attention output gate
    ``* sigmoid(gate)`` (q_proj's second half), fused into the attention kernel's store, and
    the GDN output norm ``Qwen3_5RMSNormGated(o, z)`` (z = the z projection) as the
    ``oq_rmsnorm_gated`` kernel right after the GDN step, in place.  The norm fused into the
    GDN kernel (``oq_gdn_recurrent_norm``) measured slower on B200 in this step: its
    end-of-CTA hand-off lengthens every CTA of the ~5.5-wave launch.
    """

    CONV_KERNEL = 4

    KV_BYTES_PER_TOKEN_HEAD = 264  # INT4: 2 x 128 B codes + 4 x 2 B fp16 scale/min (INT8: 520)

    def __init__(self, shape: HybridShape, *, device="cuda", seed: int = 1, page_seed: int | None = 1,
                 hold_context: bool = True, extra_tokens: int = 0, dtype=torch.bfloat16,
                 conv: str | None = None, epilogues: bool = False, kv_bits: int = 4, gates: str = "given",
                 fused_append: bool = True, early_attention: bool = True):
        # fused_append: each attention layer's launch quantises the step's new token into the
        # cache itself (oq_decode_attn_paged_append) instead of a separate append launch;
        # early_attention: an attention launch right after a GDN layer starts early and loads
        # its cached pages during that layer's tail (OQ_ATTN_EARLY: GDN launches write no cache data)
        self.fused_append = fused_append
        self.early_attention = early_attention
        # a GDN step right after an attention launch may also start early and load its state on
        # the SMs the attention leaves idle (that launch writes no GDN state): step 0.6490 ->
        # 0.6458 ms at B=64, context 4096
        self.early_gdn_after_attn = early_attention
        if conv not in (None, "separate", "fused"):
            raise ValueError("conv must be None, 'separate' or 'fused'")
        if gates not in ("given", "fused") or (gates == "fused" and conv):
            raise ValueError("gates must be 'given' or 'fused' (the latter without a conv mode)")
        self.fused_gates = gates == "fused"
        if kv_bits not in (4, 8):
            raise ValueError("kv_bits must be 4 or 8")
        self.kv_bits = kv_bits
        # K + V codes and the four fp16 scale / min values of one token and KV head
        self.kv_bytes_per_token_head = 2 * shape.head_dim * kv_bits // 8 + 8
        self.shape = shape
        self.conv = conv
        self.epilogues = epilogues
        self.device = torch.device(device)
        self.dtype = dtype
        self.hold_context = hold_context
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(seed)
        lengths = shape.lengths
        b = shape.batch
        self.attn: list[_AttnLayer] = []
        self.gdn: list[_GdnLayer] = []
        self.order: list[tuple[str, int]] = []
        for kind in shape.layer_types:
            if kind == "full_attention":
                self.order.append(("attn", len(self.attn)))
                self.attn.append(self._make_attn_layer(lengths, extra_tokens, page_seed))
            else:
                self.order.append(("gdn", len(self.gdn)))
                state = torch.randn((b, shape.gdn_heads, shape.gdn_dim, shape.gdn_dim), generator=self.gen,
                                    device=self.device, dtype=torch.float32).mul_(0.02)
                layer = _GdnLayer(state=state)
                if self.fused_gates:  # A = exp(A_log) = 1 and dt_bias = 0: g = -softplus(a), a ~ N(0, 1)
                    layer.A_log = torch.zeros(shape.gdn_heads, dtype=dtype, device=self.device)
                    layer.dt_bias = torch.zeros(shape.gdn_heads, dtype=dtype, device=self.device)
                if epilogues:
                    layer.norm_w = (1.0 + 0.1 * torch.randn(shape.gdn_dim, generator=self.gen,
                                                            device=self.device)).to(dtype)
                if conv:
                    ch = self.conv_channels
                    rnd = lambda *shp: torch.randn(shp, generator=self.gen, device=self.device)  # noqa: E731
                    layer.conv_state = rnd(b, ch, self.CONV_KERNEL).to(dtype)
                    layer.conv_w = (0.5 * rnd(ch, self.CONV_KERNEL)).to(dtype)
                    layer.conv_b = (0.1 * rnd(ch)).to(dtype)
                self.gdn.append(layer)
        self._alloc_io()
        self.graph: torch.cuda.CUDAGraph | None = None
        self.io_graph: torch.cuda.CUDAGraph | None = None
        self.stream = torch.cuda.Stream(self.device)

    @property
    def conv_channels(self) -> int:
        return self.shape.gdn_heads * 3 * self.shape.gdn_dim

    # ------------------------------------------------------------------ setup
    def _make_attn_layer(self, lengths, extra_tokens, page_seed) -> _AttnLayer:
        s = self.shape
        need = [cabi.pages_for(n + 1 + extra_tokens, s.page_size) for n in lengths]
        pool = cabi.PagedKvPool(sum(need), s.num_kv_heads, s.head_dim, s.page_size, self.device, bits=self.kv_bits)
        paged = PagedKvState(pool, s.batch, max_pages=max(need), allocator=PageAllocator(sum(need), page_seed))
        paged.reserve([n + 1 + extra_tokens for n in lengths])
        # populate each sequence's history with bf16 N(0,1) K/V, quantised by the append kernel itself;
        # rows of equal length are appended together, in token chunks of bounded size
        by_len: dict[int, list[int]] = {}
        for r, n in enumerate(lengths):
            by_len.setdefault(int(n), []).append(r)
        for n, rows in sorted(by_len.items()):
            idx = torch.tensor(rows, dtype=torch.long, device=self.device)
            table = paged.block_table.index_select(0, idx).contiguous()
            lens = torch.zeros(len(rows), dtype=torch.int32, device=self.device)
            chunk = max(1, (1 << 26) // (len(rows) * s.num_kv_heads * s.head_dim))
            for lo in range(0, n, chunk):
                m = min(chunk, n - lo)
                shp = (len(rows), s.num_kv_heads, m, s.head_dim)
                k = torch.randn(shp, generator=self.gen, device=self.device, dtype=torch.float32).to(self.dtype)
                v = torch.randn(shp, generator=self.gen, device=self.device, dtype=torch.float32).to(self.dtype)
                cabi.append_quant(k, v, pool, table, lens, advance=True)
                del k, v
            paged.seq_lens.index_copy_(0, idx, lens)
        torch.cuda.synchronize(self.device)
        paged.host_lens = list(lengths)
        write_pos = torch.tensor(lengths, dtype=torch.int32, device=self.device)
        attend = write_pos + 1
        if not self.hold_context:
            write_pos = paged.seq_lens
            attend = paged.seq_lens
        ws = cabi.new_decode_workspace(s.batch, s.num_heads, s.num_kv_heads, paged.max_pages, self.device)
        return _AttnLayer(paged=paged, write_pos=write_pos, attend_lens=attend, workspace=ws)

    def _alloc_io(self) -> None:
        """One flat input buffer and one flat output buffer, viewed per layer."""
        s = self.shape
        self._esize = torch.tensor([], dtype=self.dtype).element_size()
        b = s.batch
        in_specs, out_specs = [], []
        self._conv_out: list[torch.Tensor] = []
        for kind, i in self.order:
            if kind == "attn":
                in_specs += [(("attn", i, "q"), (b, s.num_heads, s.head_dim)),
                             (("attn", i, "k"), (b, s.num_kv_heads, 1, s.head_dim)),
                             (("attn", i, "v"), (b, s.num_kv_heads, 1, s.head_dim))]
                if self.epilogues:
                    in_specs += [(("attn", i, "gate"), (b, s.num_heads, s.head_dim))]
                out_specs += [(("attn", i, "out"), (b, s.num_heads, s.head_dim))]
            else:
                shp = (b, 1, s.gdn_heads, s.gdn_dim)
                if self.conv:
                    in_specs += [(("gdn", i, "qkv"), (b, self.conv_channels))]
                    if self.conv == "separate":  # the conv kernel's output, read by the GDN step
                        self._conv_out.append(torch.empty((b, self.conv_channels, 1), dtype=self.dtype,
                                                          device=self.device))
                else:
                    in_specs += [(("gdn", i, "q"), shp), (("gdn", i, "k"), shp), (("gdn", i, "v"), shp)]
                if not self.fused_gates:
                    in_specs += [(("gdn", i, "beta"), (b, 1, s.gdn_heads))]
                    # g stays fp32 (the module computes it in fp32): its bits take two 16-bit slots
                    # per value inside the layer's input range, so the layer's inputs are one copy
                    in_specs += [(("gdn", i, "g_bits"), (b * s.gdn_heads * 4 // self._esize,))]
                else:
                    in_specs += [(("gdn", i, "a"), (b, 1, s.gdn_heads)), (("gdn", i, "b"), (b, 1, s.gdn_heads))]
                if self.epilogues:
                    in_specs += [(("gdn", i, "z"), shp)]
                out_specs += [(("gdn", i, "out"), shp)]
        n_in = sum(math.prod(shp) for _, shp in in_specs)
        n_out = sum(math.prod(shp) for _, shp in out_specs)
        # each layer's inputs and outputs are contiguous ranges of the flat buffers (the
        # host-facing step copies them layer by layer)
        self._in_range: dict = {}
        self._out_range: dict = {}
        for specs, ranges in ((in_specs, self._in_range), (out_specs, self._out_range)):
            off = 0
            for (kind, i, _), shp in specs:
                lo, hi = ranges.get((kind, i), (off, off))
                ranges[(kind, i)] = (lo, off + math.prod(shp))
                off += math.prod(shp)
        self.in_dev = torch.empty(n_in, dtype=self.dtype, device=self.device)
        self.out_dev = torch.empty(n_out, dtype=self.dtype, device=self.device)
        self.in_host = torch.empty(n_in, dtype=self.dtype, pin_memory=True)
        self.out_host = torch.empty(n_out, dtype=self.dtype, pin_memory=True)
        off = 0
        self._g_host: list[torch.Tensor] = []
        for (kind, i, name), shp in in_specs:
            assert off % 2 == 0  # every range starts 4-byte aligned (the fp32 g views need it)
            view = self.in_dev[off:off + math.prod(shp)].view(shp)
            if name == "g_bits":
                self.gdn[i].g = view.view(torch.float32).view(b, 1, s.gdn_heads)
                self._g_host.append(self.in_host[off:off + math.prod(shp)].view(torch.float32))
            else:
                setattr((self.attn if kind == "attn" else self.gdn)[i], name, view)
            off += math.prod(shp)
        off = 0
        for (kind, i, name), shp in out_specs:
            view = self.out_dev[off:off + math.prod(shp)].view(shp)
            setattr((self.attn if kind == "attn" else self.gdn)[i], name, view)
            off += math.prod(shp)

    def fill_inputs(self) -> None:
        """Synthetic step inputs with the config-0 distributions (q/k/v bf16 N(0,1), beta = sigmoid(N),
        g = -softplus(N)), written to the pinned host buffers and the device buffers."""
        gen = torch.Generator().manual_seed(12345)
        self.in_host.copy_(torch.randn(self.in_host.shape, generator=gen).to(self.dtype))
        for gh in self._g_host:
            gh.copy_(-torch.nn.functional.softplus(torch.randn(gh.shape, generator=gen)))
        self.in_dev.copy_(self.in_host)
        for layer in self.gdn:
            if layer.beta is not None:
                layer.beta.copy_(torch.sigmoid(layer.beta.float()).to(self.dtype))
        self.in_host.copy_(self.in_dev)

    # ------------------------------------------------------------------ the step
    def step_device(self, kinds=("attn", "gdn", "append"), before=None, after=None) -> None:
        """Enqueue one step's launches; `before` / `after` (optional) are called with each
        layer's (kind, index) around its launches."""
        s = self.shape
        scaling = s.head_dim ** -0.5
        prev = None  # (kind, index) of the previous launch in this step
        for kind, i in self.order:
            if before is not None:
                before((kind, i))
            if kind == "attn":
                layer = self.attn[i]
                p = layer.paged
                if self.fused_append:
                    # one launch: the new token into the cache at write_pos, then attention over it
                    if "attn" in kinds:
                        early = self.early_attention and prev is not None and prev[0] == "gdn"
                        cabi.decode_attention(layer.q, p.pool, p.block_table, layer.write_pos, scaling,
                                              out=layer.out, workspace=layer.workspace, gate=layer.gate,
                                              new_key=layer.k[:, :, 0], new_value=layer.v[:, :, 0], early=early)
                        if not self.hold_context:
                            cabi.advance_seq_lens(p.seq_lens)
                        prev = ("attn", i)
                else:
                    if "append" in kinds:
                        cabi.append_quant(layer.k, layer.v, p.pool, p.block_table, layer.write_pos,
                                          advance=not self.hold_context)
                        prev = ("append", i)
                    if "attn" in kinds:
                        cabi.decode_attention(layer.q, p.pool, p.block_table, layer.attend_lens, scaling,
                                              out=layer.out, workspace=layer.workspace, gate=layer.gate)
                        prev = ("attn", i)
            elif "gdn" in kinds:
                layer = self.gdn[i]
                # A layer's state is written only by its own launch one step earlier, so when the
                # launch right before this one is another layer's GDN step, this one may start
                # early and load its state during that step's tail.
                # (the launch right before may also be the previous GDN layer's output norm, which
                # writes that layer's output, not this layer's state)
                chained = prev is not None and ((prev[0] == "gdn" and prev[1] != i)
                                                or (prev[0] == "attn" and self.early_gdn_after_attn))
                if self.conv == "fused":
                    cabi.gdn_conv_step(layer.qkv, layer.conv_state, layer.conv_w, layer.conv_b, layer.g, layer.beta,
                                       num_heads=s.gdn_heads, initial_state=layer.state, final_state=layer.state,
                                       out=layer.out, prefetch_state=chained)
                elif self.conv == "separate":
                    y = self._conv_out[i]
                    cabi.causal_conv1d_update(layer.qkv.unsqueeze(-1), layer.conv_state, layer.conv_w, layer.conv_b,
                                              out=y)
                    hd = s.gdn_heads * s.gdn_dim
                    q, k, v = (y[:, j * hd:(j + 1) * hd, 0].view(s.batch, 1, s.gdn_heads, s.gdn_dim) for j in range(3))
                    cabi.gdn_recurrent(q, k, v, layer.g, layer.beta, initial_state=layer.state,
                                       final_state=layer.state, out=layer.out, use_qk_l2norm=True)
                elif self.fused_gates:
                    cabi.gdn_recurrent_gates(layer.q, layer.k, layer.v, layer.a, layer.b, layer.A_log,
                                             layer.dt_bias, initial_state=layer.state, final_state=layer.state,
                                             out=layer.out, use_qk_l2norm=True, prefetch_state=chained)
                else:
                    cabi.gdn_recurrent(layer.q, layer.k, layer.v, layer.g, layer.beta, initial_state=layer.state,
                                       final_state=layer.state, out=layer.out, use_qk_l2norm=True,
                                       prefetch_state=chained)
                if layer.z is not None:
                    cabi.rmsnorm_gated(layer.out, layer.z, layer.norm_w, 1e-6, out=layer.out)
                prev = ("gdn", i)
            if after is not None:
                after((kind, i))

    def capture(self, kinds=("attn", "gdn", "append")) -> torch.cuda.CUDAGraph:
        """Capture one step's launches in a CUDA graph (after one eager warm-up step)."""
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.step_device(kinds)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self.step_device(kinds)
        return graph

    def capture_io(self, kinds=("attn", "gdn", "append")) -> torch.cuda.CUDAGraph:
        """The host-facing step as one graph with its transfers: a copy stream brings the
        inputs (and g) from the pinned host buffers in layer order, in groups of 1, 2, 4, 8,
        ... layers (one copy per group; a layer's launches wait for its group), and a second
        copy stream returns the outputs in groups that shrink toward the end (..., 2, 1
        layers).  The copies of
        later layers run under the kernels of earlier ones.  (Measured at B = 64: host-to-
        device copies slow to about a third of their idle rate while the step's kernels load
        HBM, so the compute can catch up with them; growing groups beat one copy per layer,
        and splitting the copies over more streams is slower.)  ``kinds=()`` keeps the transfers
        and drops the kernels (a measure of what the host's copies alone cost)."""
        dev = self.device
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):  # eager warm-up of the launches
            self.step_device(kinds)
        torch.cuda.current_stream(dev).wait_stream(self.stream)
        copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            main = self.stream
            fork = torch.cuda.Event()
            fork.record(main)
            copy_in.wait_event(fork)
            copy_out.wait_event(fork)
            ready = {}
            order = list(self.order)
            groups, i, n = [], 0, 1
            while i < len(order):
                groups.append(order[i:i + n])
                i, n = i + n, 2 * n
            with torch.cuda.stream(copy_in):
                for grp in groups:
                    lo, hi = self._in_range[grp[0]][0], self._in_range[grp[-1]][1]
                    self.in_dev[lo:hi].copy_(self.in_host[lo:hi], non_blocking=True)  # (g included)
                    ready[grp[0]] = torch.cuda.Event()
                    ready[grp[0]].record(copy_in)

            def before(key):
                if key in ready:
                    main.wait_event(ready[key])

            # outputs go back in groups that shrink toward the end (..., 4, 2, 1 layers), so
            # that the copy left after the last kernel is one layer's
            out_last, i, n = set(), len(order) - 1, 1
            while i >= 0:
                out_last.add(order[i])
                i, n = i - n, 2 * n
            pending = []

            def after(key):
                pending.append(key)
                if key not in out_last:
                    return
                done = torch.cuda.Event()
                done.record(main)
                copy_out.wait_event(done)
                with torch.cuda.stream(copy_out):
                    lo, hi = self._out_range[pending[0]][0], self._out_range[pending[-1]][1]
                    self.out_host[lo:hi].copy_(self.out_dev[lo:hi], non_blocking=True)
                pending.clear()

            self.step_device(kinds, before=before, after=after)
            main.wait_stream(copy_in)
            main.wait_stream(copy_out)
        return graph

    def step(self) -> torch.Tensor:
        """Host-facing step: pinned inputs -> device, the step's kernels, outputs -> the pinned
        host buffer, as one graph replay on the current stream (transfers overlap the kernels
        layer by layer).  The caller synchronises before reading the returned buffer."""
        if self.io_graph is None:
            self.io_graph = self.capture_io()
        self.io_graph.replay()
        return self.out_host

    # ------------------------------------------------------------------ accounting
    def counts(self) -> StepCounts:
        s = self.shape
        lengths = np.array(s.lengths)
        attend = lengths + 1 if self.hold_context else lengths
        attn_bytes_layer = int(attend.sum()) * s.num_kv_heads * self.kv_bytes_per_token_head
        gdn_bytes_layer = 2 * s.batch * s.gdn_heads * s.gdn_dim * s.gdn_dim * 4
        if self.conv:  # conv state read + written, plus the weights
            esz = torch.tensor([], dtype=self.dtype).element_size()
            gdn_bytes_layer += (2 * s.batch * self.conv_channels * self.CONV_KERNEL
                                + self.conv_channels * (self.CONV_KERNEL + 1)) * esz
        if self.epilogues:  # gate / z reads and the norm weight (model dtype)
            esz = torch.tensor([], dtype=self.dtype).element_size()
            attn_bytes_layer += s.batch * s.num_heads * s.head_dim * esz
            gdn_bytes_layer += (s.batch * s.gdn_heads + 1) * s.gdn_dim * esz
        append_bytes_layer = s.batch * s.num_kv_heads * (2 * s.head_dim * 2 + self.kv_bytes_per_token_head)
        n_attn, n_gdn = len(self.attn), len(self.gdn)
        esize = self.in_dev.element_size()
        attn_launches = (1 + (0 if self.hold_context else 1)) if self.fused_append else 2
        per_kernel = {"gdn_recurrent": gdn_bytes_layer}
        if self.fused_append:  # the attention launch also reads the new token and writes its codes
            per_kernel[f"decode_attn_int{self.kv_bits}_paged"] = attn_bytes_layer + append_bytes_layer
        else:
            per_kernel[f"decode_attn_int{self.kv_bits}_paged"] = attn_bytes_layer
            per_kernel[f"append_quant_int{self.kv_bits}"] = append_bytes_layer
        return StepCounts(
            launches=attn_launches * n_attn
            + n_gdn * ((2 if self.conv == "separate" else 1) + (1 if self.epilogues else 0)),
            attn_bytes=attn_bytes_layer * n_attn,
            gdn_bytes=gdn_bytes_layer * n_gdn,
            append_bytes=append_bytes_layer * n_attn,
            h2d_bytes=self.in_dev.numel() * esize,
            d2h_bytes=self.out_dev.numel() * esize,
            per_kernel=per_kernel,
        )
