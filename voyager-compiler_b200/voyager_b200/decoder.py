"""LLaMA-style decoder stack over the quantized ops (benchmark config C5).

This is the forward that a PT2E-converted LLaMA graph runs when every linear
and both attention matmuls are MXFP8 (``fp8_e4m3,qs=microscaling,bs=32`` with
``force_scale_power_of_two``): ``convert_pt2e`` quantizes each weight once
(``src/voyager_compiler/quantize_pt2e.py:739-766``), inserts a
``quantize_mx`` before every activation operand (``:779-808``) with blocks
along the operand's contraction axis (``:136-161``: -1 for a matmul's first
operand, -2 for its second), and retargets ``linear`` / ``matmul`` to
``linear_mx`` / ``matmul_mx`` (``:851-938``).  Everything between those ops
(RMSNorm, RoPE, softmax, SwiGLU, residual adds) stays in bf16 torch ops, as
in the exported eager graph of HF LLaMA.

Two rewrites that leave every value unchanged:
  * q/k/v and gate/up share their input codes, so each group is one
    ``linear_mx`` over the concatenated weight rows (every output element is
    the same dot product over the same K blocks);
  * the second operand of ``q @ k^T`` is quantized as ``k`` along its last
    axis and passed transposed (a block of 32 along -2 of ``k^T`` is the same
    32 values as a block along -1 of ``k``); likewise ``v``'s blocks along the
    token axis are computed on ``v^T`` along -1.
The attention itself is either ``sdpa_mx`` (a model exported with
scaled-dot-product attention; ``quantize_pt2e`` converts it to this op) or
the eager matmul / softmax graph; they differ only in where the masked
scores are set to -inf (``masked_fill`` vs. adding the dtype's minimum), and
both give the masked keys a probability of exactly 0.

Tensor parallel (Megatron with sequence-parallel norms) when a process group
of g > 1 ranks is given: the residual stream is split by tokens; q/k/v and
gate/up are column-parallel (output rows / heads split g ways), o_proj and
down row-parallel (K split g ways at multiples of 32, so every quantization
block of the single-device graph stays whole on one rank).  Per layer: the
normalised activations are quantized on their token shard and all-gathered
(codes + scales, bit-identical to quantizing the full tensor), and the
row-parallel partial products are reduce-scattered back to token shards.

Weights are random-init N(0, 0.02) (no checkpoint); ``init_weights`` makes
them from a seed so every rank (and a CPU check) builds the same model.
"""

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

W_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass
class DecoderConfig:
    layers: int = 4
    hidden: int = 4096
    heads: int = 32
    ffn: int = 11008
    eps: float = 1e-5
    rope_theta: float = 10000.0
    block_size: int = 32

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def flops(self, batch: int, seq: int) -> float:
        """Forward FLOPs of the matmuls as the eager graph computes them
        (full S x S attention products)."""
        t = batch * seq
        lin = 2 * t * self.hidden * (4 * self.hidden + 3 * self.ffn)
        att = 2 * 2 * batch * self.heads * seq * seq * self.head_dim
        return float(self.layers * (lin + att))


def init_weights(cfg: DecoderConfig, seed: int, device) -> List[Dict[str, torch.Tensor]]:
    """bf16 weights ~ N(0, 0.02) per layer ([out, in] like nn.Linear), the
    RMSNorm weights ones; drawn in a fixed order from one generator."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    h, f = cfg.hidden, cfg.ffn
    shapes = {"q": (h, h), "k": (h, h), "v": (h, h), "o": (h, h),
              "gate": (f, h), "up": (f, h), "down": (h, f)}
    layers = []
    for _ in range(cfg.layers):
        w = {n: (torch.randn(shapes[n], generator=gen, device=device) * 0.02).bfloat16()
             for n in W_NAMES}
        w["ln1"] = torch.ones(h, dtype=torch.bfloat16, device=device)
        w["ln2"] = torch.ones(h, dtype=torch.bfloat16, device=device)
        layers.append(w)
    return layers


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """LLaMA RMSNorm: float32 statistics, cast back to the input dtype, times
    the weight."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(x.dtype)


def rope_tables(seq: int, dim: int, theta: float, device, dtype):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64, device=device).float() / dim))
    t = torch.arange(seq, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [B, heads, S, D]; the rotate-half convention of HF LLaMA."""
    d = x.shape[-1] // 2
    rot = torch.cat([-x[..., d:], x[..., :d]], dim=-1)
    return x * cos + rot * sin


class TensorParallel:
    """The process group a decoder is split over (world 1: no collectives)."""

    def __init__(self, group=None, enabled: bool = True):
        on = enabled and dist.is_available() and dist.is_initialized()
        self.group = group
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0

    def split(self, n: int, what: str) -> slice:
        if n % self.world:
            raise ValueError(f"{what}: {n} does not split into {self.world} equal shards")
        step = n // self.world
        return slice(self.rank * step, (self.rank + 1) * step)

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        t = t.contiguous()
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                          device=t.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        return out

    def reduce_scatter_rows(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        t = t.contiguous()
        out = torch.empty((t.shape[0] // self.world,) + tuple(t.shape[1:]), dtype=t.dtype,
                          device=t.device)
        dist.reduce_scatter_tensor(out, t, group=self.group)
        return out


class DecoderLayer:
    def __init__(self, cfg: DecoderConfig, w: Dict[str, torch.Tensor], table: torch.Tensor,
                 ops, tp: TensorParallel, attn: str = "sdpa", fused: bool = False):
        if attn not in ("sdpa", "eager"):
            raise ValueError(f"attn must be 'sdpa' or 'eager', not {attn!r}")
        self.cfg, self.table, self.ops, self.tp, self.attn = cfg, table, ops, tp, attn
        self.fused = fused
        h, f = cfg.hidden, cfg.ffn
        if cfg.heads % tp.world:
            raise ValueError(f"{cfg.heads} heads do not split over {tp.world} ranks")
        hs = tp.split(h, "hidden")
        fs = tp.split(f, "ffn")
        for n, k in ((h // tp.world, "hidden shard"), (f // tp.world, "ffn shard")):
            if n % cfg.block_size or n % 8:
                raise ValueError(f"{k} {n} is not a multiple of the block size and of 8")
        self.ln1, self.ln2 = w["ln1"], w["ln2"]
        # column-parallel: this rank's output rows; row-parallel: its K columns
        qkv = torch.cat([w["q"][hs], w["k"][hs], w["v"][hs]], 0)
        gu = torch.cat([w["gate"][fs], w["up"][fs]], 0)
        self.qkv = self._quant_weight(qkv)
        self.gu = self._quant_weight(gu)
        self.o = self._quant_weight(w["o"][:, hs])
        self.down = self._quant_weight(w["down"][:, fs])

    def _qmx(self, x: torch.Tensor):
        """quantize_mx along the last axis (MXFP8, power-of-two scales)."""
        return self.ops.quantize_mx(x, self.table, [-1], self.cfg.block_size, 448.0, True)

    def _quant_weight(self, w: torch.Tensor):
        scale, codes = self._qmx(w.contiguous())
        return codes, scale

    def _linear(self, codes, scale, w):
        return self.ops.linear_mx(codes, w[0], None, input_scale=scale, weight_scale=w[1],
                                  block_size=self.cfg.block_size)

    def _linear_add(self, codes, scale, w, x):
        """x + linear_mx(...): on one GPU with this library's ops, the add is
        done by the GEMM epilogue (bf16(linear) + x, the same two roundings);
        otherwise the row-parallel product is reduce-scattered and added."""
        if self.fused and self.tp.world == 1 and isinstance(self.ops, _CudaOps):
            from voyager_b200 import mxgemm

            if mxgemm.applies(codes, w[0], scale, w[1], self.cfg.block_size, None, None, "kc",
                              "linear"):
                out = mxgemm.linear(codes, w[0], None, scale, w[1], residual=x.contiguous())
                if out is not None:
                    return out
        return x + self.tp.reduce_scatter_rows(self._linear(codes, scale, w))

    def _gathered_qmx(self, x: torch.Tensor, norm_w: Optional[torch.Tensor] = None):
        """quantize_mx of the token shard (RMSNorm'd first when ``norm_w`` is
        given), then all-gather codes and scales."""
        if norm_w is None:
            scale, codes = self._qmx(x)
        elif self.fused:
            from voyager_b200 import fused

            scale, codes = fused.rmsnorm_quantize_mx(x, norm_w, self.cfg.eps, self.table)
        else:
            scale, codes = self._qmx(rms_norm(x, norm_w, self.cfg.eps))
        codes = self.tp.all_gather_rows(codes)
        scale = self.tp.all_gather_rows(scale)
        mark = getattr(self.ops, "mark_exact", None)
        if mark is not None and self.tp.world > 1:
            mark(codes, scale)
        return codes, scale

    def __call__(self, x: torch.Tensor, batch: int, cos, sin, mask) -> torch.Tensor:
        """x: this rank's token shard [T/g, H] of the [batch * S, H] residual
        stream -> the same shard after the layer."""
        cfg, tp, ops = self.cfg, self.tp, self.ops
        bs = cfg.block_size
        T = x.shape[0] * tp.world
        S = T // batch
        nh, hd = cfg.heads // tp.world, cfg.head_dim
        hl = nh * hd
        # --- attention ---------------------------------------------------
        codes, scale = self._gathered_qmx(x, self.ln1)
        qkv = self._linear(codes, scale, self.qkv)                    # [T, 3 hl]
        if self.fused and S % 128 == 0:
            from voyager_b200 import fused

            (sq, cq), (sk, ck) = fused.rope_quantize_qk(qkv, 0, hl, cos, sin, batch, S, nh,
                                                        self.table)
            sv, cv = fused.quantize_vt(qkv, 2 * hl, batch, S, nh, self.table)
        else:
            q, k, v = (t.reshape(batch, S, nh, hd).transpose(1, 2) for t in qkv.split(hl, -1))
            q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
            sq, cq = self._qmx(q.contiguous())
            sk, ck = self._qmx(k.contiguous())
            sv, cv = self._qmx(v.transpose(-1, -2).contiguous())
        if self.attn == "sdpa":
            # scaled_dot_product_attention(is_causal=True), converted
            o = ops.sdpa_mx(cq, ck, cv.transpose(-1, -2), is_causal=True, query_scale=sq,
                            key_scale=sk, value_scale=sv.transpose(-1, -2), block_size=bs,
                            probs_qmap=self.table, probs_quant_max=448.0,
                            force_scale_power_of_two=True)
        else:
            # eager attention: matmul, scale, additive mask, float32 softmax
            scores = ops.matmul_mx(cq, ck.transpose(-1, -2), input_scale=sq,
                                   weight_scale=sk.transpose(-1, -2), block_size=bs)
            scores = scores * (1.0 / math.sqrt(hd)) + mask
            probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(x.dtype)
            sp, cp = self._qmx(probs)
            o = ops.matmul_mx(cp, cv.transpose(-1, -2), input_scale=sp,
                              weight_scale=sv.transpose(-1, -2), block_size=bs)
        o = o.transpose(1, 2).reshape(T, hl)
        so, co = self._qmx(o)
        x = self._linear_add(co, so, self.o, x)
        # --- SwiGLU MLP ----------------------------------------------------
        codes, scale = self._gathered_qmx(x, self.ln2)
        gu = self._linear(codes, scale, self.gu)
        if self.fused:
            from voyager_b200 import fused

            sa, ca = fused.swiglu_quantize_mx(gu, gu.shape[-1] // 2, self.table)
        else:
            g, u = gu.chunk(2, -1)
            sa, ca = self._qmx(torch.nn.functional.silu(g) * u)
        return self._linear_add(ca, sa, self.down, x)


class ColumnParallelLayer:
    """A decoder layer with every linear split by output features over the
    group (column parallel) and the residual stream split by hidden columns:
    rank r holds x[:, r*H/g:(r+1)*H/g] for all tokens, the q/k/v rows of its
    H/g / 128 heads, o_proj's and down's output rows of its hidden columns
    and gate/up's rows of its ffn columns.  Every GEMM sums over its full K,
    so each output value is the one-GPU value; the only cross-rank arithmetic
    is RMSNorm's row statistic, summed from the ranks' partial sums in rank
    order.  Each linear's input -- the normalised activations (twice), the
    attention output and the SwiGLU activation -- is quantized by the rank
    that owns its columns and written straight into every rank's copy of the
    full-width MXFP8 operand through NVLS multicast (``voyager_b200.tp``);
    one barrier follows each such write, six per layer."""

    def __init__(self, cfg: DecoderConfig, w: Dict[str, torch.Tensor], table: torch.Tensor,
                 tp: TensorParallel):
        from voyager_b200.tp import pad_k_chunks

        g, r = tp.world, tp.rank
        h, f = cfg.hidden, cfg.ffn
        if cfg.heads % g or h % g or f % g:
            raise ValueError(f"heads / hidden / ffn do not split over {g} ranks")
        self.hs, self.fs = h // g, f // g
        if self.hs % 128 or self.fs % 32:
            raise ValueError(f"hidden shard {self.hs} (multiple of 128) or ffn shard {self.fs} "
                             "(multiple of 32) does not fit the MXFP8 operand tiles")
        self.fs_p = (self.fs + 127) // 128 * 128
        self.cfg, self.table, self.tp = cfg, table, tp
        hsl, fsl = slice(r * self.hs, (r + 1) * self.hs), slice(r * self.fs, (r + 1) * self.fs)
        self.ln1 = w["ln1"][hsl].contiguous()
        self.ln2 = w["ln2"][hsl].contiguous()
        q = torch.ops.quantized_ops

        def quant(wt):
            s_, c_ = q.quantize_mx(wt.contiguous(), table, [-1], cfg.block_size, 448.0, True)
            return c_, s_

        self.qkv = quant(torch.cat([w["q"][hsl], w["k"][hsl], w["v"][hsl]], 0))
        self.o = quant(w["o"][hsl])
        self.gu = quant(torch.cat([w["gate"][fsl], w["up"][fsl]], 0))
        self.down = quant(pad_k_chunks(w["down"][hsl], g))

    def operands(self) -> Dict[str, int]:
        h = self.cfg.hidden
        return {"h1": h, "o": h, "h2": h, "act": self.tp.world * self.fs_p}

    def _gemm(self, ws, name, wq, out, residual=None):
        from voyager_b200 import mxgemm
        from voyager_b200.ops import _stream

        K, a_p, a_s, _, _ = ws.operand(name)
        pw, pws, ok = mxgemm.packed_weight(wq[0], wq[1])
        if not ok:
            raise RuntimeError("column-parallel decoder: weight operand is not exact MXFP8")
        N = wq[0].shape[0]
        st = _lib().vq_gemm_mxf8_ex(
            a_p, a_s, pw.data_ptr(), pws.data_ptr(), ws.T, N, K, None,
            None if residual is None else residual.data_ptr(), N, out.data_ptr(), N, 0,
            ws.gemm_err.data_ptr(), _stream(out.device))
        _check(st, "column-parallel decoder GEMM")

    def _norm(self, ws, x, weight, name, rd, fl2q, stream):
        lib = _lib()
        _check(lib.vq_tp_sumsq(x.data_ptr(), ws.T, self.hs, ws.stats_mc(), ws.rank, stream),
               "tp sumsq")
        ws.barrier(stream)
        _, _, _, p_mc, a_mc = ws.operand(name)
        _check(lib.vq_tp_norm_quantize(x.data_ptr(), ws.T, self.hs, ws.stats_local(), ws.world,
                                       self.cfg.hidden, weight.data_ptr(), float(self.cfg.eps),
                                       rd.ref(), fl2q, p_mc, a_mc, self.cfg.hidden,
                                       ws.rank * self.hs, ws.RT, stream), "tp norm quantize")
        ws.barrier(stream)

    def __call__(self, x: torch.Tensor, ws, batch: int, cos, sin) -> torch.Tensor:
        """x: [T, H/g], this rank's hidden columns (updated in place)."""
        from voyager_b200 import fused
        from voyager_b200.ops import _stream, floor_log2
        from voyager_b200.tables import rounder_for

        cfg, g = self.cfg, self.tp.world
        T, dev = x.shape[0], x.device
        S, nh, hs = T // batch, cfg.heads // g, self.hs
        stream = _stream(dev)
        rd = rounder_for(self.table, dev)
        fl2q = floor_log2(448.0)
        lib = _lib()
        # attention block
        self._norm(ws, x, self.ln1, "h1", rd, fl2q, stream)
        qkv = torch.empty((T, 3 * hs), dtype=torch.bfloat16, device=dev)
        self._gemm(ws, "h1", self.qkv, qkv)
        (sq, cq), (sk, ck) = fused.rope_quantize_qk(qkv, 0, hs, cos, sin, batch, S, nh, self.table)
        sv, cv = fused.quantize_vt(qkv, 2 * hs, batch, S, nh, self.table)
        o = torch.ops.quantized_ops.sdpa_mx(
            cq, ck, cv.transpose(-1, -2), is_causal=True, query_scale=sq, key_scale=sk,
            value_scale=sv.transpose(-1, -2), block_size=cfg.block_size, probs_qmap=self.table,
            probs_quant_max=448.0, force_scale_power_of_two=True)
        o = o.transpose(1, 2).reshape(T, hs)
        _, _, _, p_mc, a_mc = ws.operand("o")
        _check(lib.vq_tp_quantize(o.data_ptr(), hs, T, hs, rd.ref(), fl2q, p_mc, a_mc,
                                  cfg.hidden, ws.rank * hs, ws.RT, stream), "tp quantize")
        ws.barrier(stream)
        self._gemm(ws, "o", self.o, x, residual=x)
        # MLP block
        self._norm(ws, x, self.ln2, "h2", rd, fl2q, stream)
        gu = torch.empty((T, 2 * self.fs), dtype=torch.bfloat16, device=dev)
        self._gemm(ws, "h2", self.gu, gu)
        K, _, _, p_mc, a_mc = ws.operand("act")
        _check(lib.vq_tp_swiglu_quantize(gu.data_ptr(), 2 * self.fs, self.fs, T, self.fs,
                                         rd.ref(), fl2q, p_mc, a_mc, K, ws.rank * self.fs_p,
                                         ws.RT, stream), "tp swiglu quantize")
        ws.barrier(stream)
        self._gemm(ws, "act", self.down, x, residual=x)
        return x


def _lib():
    from voyager_b200 import _lib as L

    return L.load()


def _check(st, what):
    from voyager_b200 import _lib as L

    L.check(st, what)


class Decoder:
    """``cfg.layers`` decoder layers, tensor parallel over ``group`` (the
    default process group when one is initialised; ``parallel=False`` keeps
    the whole model on this rank; in the column split ``micro_batches``
    groups of sequences run on separate streams so that communication
    overlaps compute); ``ops`` defaults to
    ``torch.ops.quantized_ops`` (this library's CUDA kernels).  ``attn``:
    "sdpa" -- the graph of a model exported with scaled-dot-product attention,
    converted to ``sdpa_mx`` (one fused kernel); "eager" -- the eager
    attention graph (``matmul_mx``, scale, additive causal mask, float32
    softmax, ``quantize_mx`` of the probabilities, ``matmul_mx``).  Both
    compute the same values.  ``fused`` (default: with the CUDA ops) runs
    RMSNorm, RoPE, the v transpose and SwiGLU inside the quantize_mx that
    follows each of them (``voyager_b200.fused``)."""

    def __init__(self, cfg: DecoderConfig, weights: List[Dict[str, torch.Tensor]], *,
                 table: Optional[torch.Tensor] = None, ops=None, group=None,
                 attn: str = "sdpa", fused: Optional[bool] = None, parallel: bool = True,
                 tp_mode: str = "auto", micro_batches: int = 2):
        self.cfg = cfg
        self.tp = TensorParallel(group, parallel)
        self.ops = ops if ops is not None else _CudaOps()
        dev = weights[0]["q"].device
        if table is None:
            from voyager_b200.tables import get_quantization_map

            table = get_quantization_map("fp8_e4m3", dev)
        if fused is None:
            fused = isinstance(self.ops, _CudaOps)
        if tp_mode not in ("auto", "columns", "megatron"):
            raise ValueError(f"tp_mode must be auto, columns or megatron, not {tp_mode!r}")
        self.columns = False
        if self.tp.world > 1 and tp_mode != "megatron" and isinstance(self.ops, _CudaOps):
            from voyager_b200.tp import multicast_available

            self.columns = tp_mode == "columns" or (
                multicast_available(group) and attn == "sdpa" and fused
                and (cfg.hidden // self.tp.world) % 128 == 0)
        if self.columns:
            self.layers = [ColumnParallelLayer(cfg, w, table, self.tp) for w in weights]
        else:
            self.layers = [DecoderLayer(cfg, w, table, self.ops, self.tp, attn, fused)
                           for w in weights]
        self._tabs = {}
        self._ws = []
        self._streams = []
        self.micro_batches = micro_batches

    def _tables(self, seq: int, device, dtype):
        key = (seq, device, dtype)
        if key not in self._tabs:
            cos, sin = rope_tables(seq, self.cfg.head_dim, self.cfg.rope_theta, device, dtype)
            mask = torch.full((seq, seq), torch.finfo(dtype).min, dtype=dtype,
                              device=device).triu(1)
            self._tabs[key] = (cos, sin, mask)
        return self._tabs[key]

    def shard(self, flat: torch.Tensor) -> torch.Tensor:
        """The part of the [T, H] hidden states this rank's forward_shard
        takes: its token rows (Megatron split) or its hidden columns (column
        split)."""
        if self.columns:
            return flat[:, self.tp.split(flat.shape[1], "hidden")].contiguous()
        return flat[self.tp.split(flat.shape[0], "tokens")].contiguous()

    def unshard(self, y: torch.Tensor) -> torch.Tensor:
        """The full [T, H] from every rank's shard (an all-gather)."""
        if not self.columns:
            return self.tp.all_gather_rows(y)
        g = self.tp.world
        parts = self.tp.all_gather_rows(y)  # [g * T, H/g]
        T = y.shape[0]
        return parts.view(g, T, -1).permute(1, 0, 2).reshape(T, -1)

    def _workspace(self, i: int, tokens: int, device):
        """The symmetric workspace of micro-batch i (its own operand buffers
        and barrier flags, so micro-batches on different streams never wait
        on each other's flags)."""
        from voyager_b200.tp import Workspace

        while len(self._ws) <= i:
            self._ws.append(None)
        if self._ws[i] is None or self._ws[i].T != tokens:
            self._ws[i] = None
            self._ws[i] = Workspace(self.tp.group, tokens, self.layers[0].operands(), device)
            self._ws[i].gemm_err = torch.zeros(1, dtype=torch.int32, device=device)
        return self._ws[i]

    def _micro_batches(self, batch: int, tokens: int) -> int:
        """Two micro-batches (independent sequences) on two streams when the
        batch splits evenly into 128-token multiples: one half's NVLink
        stores and barrier waits overlap the other half's GEMMs."""
        n = self.micro_batches
        if n > 1 and batch % n == 0 and (tokens // n) % 128 == 0:
            return n
        return 1

    @torch.no_grad()
    def forward_shard(self, x: torch.Tensor, batch: int) -> torch.Tensor:
        """x: this rank's shard (``shard``) -> the shard after all layers."""
        if self.columns:
            T, dev = x.shape[0], x.device
            cos, sin, _ = self._tables(T // batch, dev, x.dtype)
            nb = self._micro_batches(batch, T)
            if nb == 1:
                ws = self._workspace(0, T, dev)
                x = x.clone()
                for layer in self.layers:
                    x = layer(x, ws, batch, cos, sin)
                return x
            main = torch.cuda.current_stream(dev)
            while len(self._streams) < nb:
                self._streams.append(torch.cuda.Stream(dev))
            tm = T // nb
            wss = [self._workspace(i, tm, dev) for i in range(nb)]
            start = torch.cuda.Event()
            start.record(main)
            outs = []
            for i in range(nb):
                st = self._streams[i]
                st.wait_event(start)
                with torch.cuda.stream(st):
                    xi = x[i * tm:(i + 1) * tm].clone()
                    for layer in self.layers:
                        xi = layer(xi, wss[i], batch // nb, cos, sin)
                outs.append(xi)
            for i in range(nb):
                main.wait_stream(self._streams[i])
                outs[i].record_stream(main)
            return torch.cat(outs, 0)
        S = x.shape[0] * self.tp.world // batch
        cos, sin, mask = self._tables(S, x.device, x.dtype)
        for layer in self.layers:
            x = layer(x, batch, cos, sin, mask)
        return x

    def check_errors(self):
        """Raise if a bounded device wait gave up since the workspace was made."""
        for ws in self._ws:
            if ws is not None:
                ws.check()
                if int(ws.gemm_err.item()):
                    raise RuntimeError("decoder GEMM: device wait timed out")

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: the full hidden states [B, S, H] (the same on every rank) ->
        [B, S, H]; with g > 1 ranks the output is all-gathered."""
        B, S, H = x.shape
        y = self.forward_shard(self.shard(x.reshape(B * S, H)), B)
        return self.unshard(y).reshape(B, S, H)

    __call__ = forward


class _CudaOps:
    """``torch.ops.quantized_ops`` plus ``mark_exact``: codes and scales that
    were gathered from this library's ``quantize_mx`` outputs are E4M3 values
    and powers of two by construction, so ``linear_mx`` may skip its
    operand check on them."""

    def __init__(self):
        self._q = torch.ops.quantized_ops
        self.quantize_mx = self._q.quantize_mx
        self.linear_mx = self._q.linear_mx
        self.matmul_mx = self._q.matmul_mx
        self.sdpa_mx = self._q.sdpa_mx

    @staticmethod
    def mark_exact(codes, scale):
        from voyager_b200 import mxgemm

        mxgemm.vouch(codes, scale)
