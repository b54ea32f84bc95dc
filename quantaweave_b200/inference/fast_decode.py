"""Incremental decoding with a KV cache (reference ``src/fast_decode.py``: ``FastDecoder`` :86-379,
``filter_logits`` :40-50).

Behaviour kept from the reference: no expert capacity at inference; a context of ``max_sequence_length - 1`` tokens
(learned positions) with the oldest half dropped and re-read when it fills; ``feed``/``append``/``stream``/``warm``;
greedy argmax or Gumbel-max sampling with top-k/top-p filtering. ``stream`` reads each token id back to the host
(callers check stop strings per token); ``generate`` keeps greedy tokens on the device.

B200 design:

* batched: ``generate(prompts [B, P], max_new)`` decodes B sequences together (the reference is batch-1 only);
* quantised experts stay packed (int4 g128 fp16 scales / int8 per-channel) and are dequantised in registers by the
  grouped GEMV kernel, which streams each selected expert's rows once for all tokens routed to it;
* split-K decode attention over a bf16 ``[B, Hkv, Lmax, D]`` cache (GQA heads packed per block), RoPE and the cache
  append fused in one kernel, routing by the fp32 router kernels with the capacity plan disabled;
* the whole one-token step (all layers and the LM head) is captured as one CUDA graph; every decode kernel is
  launched with programmatic dependent launch so the next kernel's weight prefetch overlaps the previous one;
* prefill runs the training kernels (tcgen05 GEMMs, flash attention, grouped SwiGLU) over the prompt.

On CPU the same step runs as plain fp32 PyTorch (the oracle the GPU path is tested against).

Expert-parallel models (the reference refuses them, ``src/fast_decode.py:89-90``) decode SPMD: every rank of the
expert group runs the same prompts and tokens through the replicated layers; at each MoE layer a rank runs only the
routes to its own experts, so every rank produces the same logits (and, with the same seed, the same samples). On
CUDA this is the native graph-captured step: the routing kernel lists only this rank's experts, the grouped GEMVs run
them, and ``csrc/ep_decode.cu`` stores each token's partial MoE output into every rank's exchange plane with NVLink
peer stores and a release flag; the next layer's norm kernel sums the planes in rank order. On CPU the partial outputs
are summed with one all-reduce (the oracle).
"""

from __future__ import annotations

import contextlib
import math
from typing import Iterator, Optional

import torch
import torch.nn.functional as F
from torch import Tensor

BATCH = 8


class Unsupported(Exception):
    """The model layout is not handled by the decoder (tensor-parallel attention, pipeline stages, ...)."""


def filter_logits(logits: Tensor, top_k: int = 0, top_p: float = 1.0) -> Tensor:
    """Top-k then nucleus filtering along the last dimension; removed entries become -inf (graph-safe)."""
    if top_k and top_k < logits.size(-1):
        threshold = torch.topk(logits, top_k, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < threshold, float("-inf"))
    if top_p < 1.0:
        sorted_logits, order = torch.sort(logits, descending=True, dim=-1)
        probs = sorted_logits.softmax(dim=-1)
        remove = probs.cumsum(dim=-1) - probs > top_p
        logits = torch.empty_like(logits).scatter_(-1, order, sorted_logits.masked_fill(remove, float("-inf")))
    return logits


def layer_weight(module) -> Tensor:
    """The dense weight a linear-like module applies (reference ``src/fast_decode.py:65-73``): a plain
    ``nn.Linear``'s weight, a LoRA projection's merged weight, or a quantised projection dequantised."""
    if isinstance(module, torch.nn.Linear):
        return module.weight.detach()
    if hasattr(module, "merged_weight"):
        return module.merged_weight()
    if hasattr(module, "dequantize"):
        return module.dequantize()
    raise Unsupported(f"cannot read the weights of {type(module).__name__}")


def precision_dtype(device: torch.device, precision: str) -> torch.dtype:
    if precision == "auto":
        precision = "bf16" if device.type == "cuda" else "fp32"
    return {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[precision]


class _Layer:
    pass


class FastDecoder:
    def __init__(self, model, device: torch.device, precision: str = "auto", use_graph: Optional[bool] = None,
                 compile: Optional[bool] = None, max_batch: int = 1, max_length: Optional[int] = None) -> None:
        from ..models.layers import Attention

        if not all(hasattr(model, name) for name in ("config", "blocks", "token_embedding", "lm_head")):
            raise Unsupported(f"{type(model).__name__} is not a QuantaWeave causal LM")
        ep = getattr(model, "expert_parallel", None)
        if getattr(model, "pipeline", None) is not None:
            raise Unsupported("pipeline-stage models hold only some layers")
        if ep is not None and (getattr(ep, "tp_size", 1) > 1 or getattr(ep, "sequence_parallel", False)):
            raise Unsupported("tensor-parallel attention")
        cfg = model.config
        self.model = model
        self.config = cfg
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:  # a concrete GPU (collectives name it)
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.ep = ep if ep is not None and ep.world_size > 1 else None
        self.native = self.device.type == "cuda"
        if self.native:
            # the prefill runs the model's own native modules: bf16 matrices, fp32 router/norms (in place)
            from ..training.native import prepare_model

            prepare_model(model, "bf16")
        self.dtype = torch.bfloat16 if self.native else precision_dtype(self.device, precision)
        self.learned = cfg.position_embedding == "learned"
        self.capacity = (cfg.max_sequence_length - 1) if self.learned else (max_length or cfg.max_sequence_length - 1)
        self.max_batch = max_batch
        self.heads, self.kv_heads, self.head_dim = cfg.attention_heads, cfg.num_kv_heads, cfg.head_dim
        self.hidden, self.vocab = cfg.hidden_size, cfg.vocab_size
        self.layers: list[_Layer] = []
        dev, dt = self.device, self.dtype
        with torch.no_grad():
            self.tok_emb = model.token_embedding.weight.detach().to(dev, dt)
            self.pos_emb = model.position_embedding.weight.detach().to(dev, dt) if self.learned else None
            self.final_norm = self._norm(model.final_norm)
            self.lm_head = self._lm_head(model.lm_head)
            for block in model.blocks:
                if not isinstance(block.attention, Attention):
                    raise Unsupported("tensor-parallel attention")
                layer = _Layer()
                att, moe = block.attention, block.moe
                layer.norm1, layer.norm2 = self._norm(block.attention_norm), self._norm(block.moe_norm)
                layer.wqkv = att.in_proj_weight.detach().to(dev, dt).contiguous()
                layer.bqkv = att.in_proj_bias.detach().to(dev, torch.float32) if att.in_proj_bias is not None else None
                layer.wo = att.out_proj.weight.detach().to(dev, dt).contiguous()
                layer.bo = att.out_proj.bias.detach().to(dev, torch.float32) if att.out_proj.bias is not None else None
                layer.router = moe.router.weight.detach().to(dev, torch.float32).contiguous()
                layer.temperature = float(moe.router_temperature)
                layer.bias = moe.expert_bias.detach().float().to(dev) if moe.expert_bias is not None else None
                layer.top_k = moe.top_k
                layer.num_experts = moe.num_experts
                layer.ffn = moe.ffn_local
                self._experts(layer, moe)
                shape = (max_batch, self.kv_heads, self.capacity, self.head_dim)
                layer.keys = torch.zeros(shape, dtype=dt, device=dev)
                layer.values = torch.zeros(shape, dtype=dt, device=dev)
                self.layers.append(layer)
        if cfg.position_embedding == "rope":
            from ..models.layers import rope_tables

            cos, sin = rope_tables(torch.arange(self.capacity + 1, device=dev), self.head_dim, cfg.rope_theta)
            self.cos, self.sin = cos.contiguous(), sin.contiguous()
        else:
            self.cos = self.sin = torch.zeros(1, device=dev)
        if self.native and self.ep is not None:
            self._setup_ep_exchange()
        # static step inputs/outputs (graph-safe)
        self.tokens_in = torch.zeros(max_batch, dtype=torch.long, device=dev)
        self.positions_in = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(max_batch, self.vocab, dtype=torch.float32, device=dev)
        self.noise = torch.zeros(BATCH, self.vocab, dtype=torch.float32, device=dev)
        self.sampled = torch.zeros(BATCH, max_batch, dtype=torch.long, device=dev)
        self.slot = torch.zeros(1, dtype=torch.long, device=dev)
        self.logit_mask = torch.zeros(self.vocab, dtype=torch.float32, device=dev)
        # ticket counters of the decode kernels whose last block finishes the work (each kernel resets its own)
        self._tickets = torch.zeros(max(max_batch * self.kv_heads, 1), dtype=torch.int32, device=dev)
        self._programs: dict = {}
        self.length = 0
        self.tokens: list[int] = []
        self.graph = None
        self.compiled = False
        self.compile_error: Optional[str] = None
        self.graph_enabled = self.native if use_graph is None else bool(use_graph and self.native)
        if self.graph_enabled:
            self._capture()

    def _setup_ep_exchange(self) -> None:
        """Symmetric buffers of the expert-parallel decode exchange (collective over the expert group): two planes per
        layer of ``[world][max_batch][hidden]`` fp32 partial outputs, one flag word per peer, a device step counter."""
        import torch.distributed as dist

        from ..parallel.p2p import P2PTransport

        ep, dev = self.ep, self.device
        transport = P2PTransport.for_group(ep.group, dev)
        symm, name = transport.symm, transport._group_name()
        local = self.layers[0].q_gu.size(0)
        self._ep_first, self._ep_local = ep.rank * local, local
        self._ep_me, self._ep_world = transport.me, transport.world
        self._ep_plane = self._ep_world * self.max_batch * self.hidden
        self._ep_parts = symm.empty(2 * len(self.layers) * self._ep_plane, dtype=torch.float32, device=dev)
        self._ep_parts.zero_()
        parts_handle = symm.rendezvous(self._ep_parts, name)
        self._ep_flags = symm.empty(self._ep_world, dtype=torch.int32, device=dev)
        self._ep_flags.zero_()
        flags_handle = symm.rendezvous(self._ep_flags, name)
        self._ep_handles = (parts_handle, flags_handle)
        self._ep_peers = torch.tensor([int(p) for p in parts_handle.buffer_ptrs], dtype=torch.int64, device=dev)
        self._ep_peer_flags = torch.tensor([int(p) for p in flags_handle.buffer_ptrs], dtype=torch.int64, device=dev)
        self._ep_step = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ep_done = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ep_timeout = transport.timeout_s
        torch.cuda.synchronize(dev)
        dist.barrier(group=ep.group, device_ids=[dev.index if dev.index is not None else torch.cuda.current_device()])

    # ---- weight extraction -----------------------------------------------------------------------
    def _norm(self, norm):
        w = norm.weight.detach().to(self.device, torch.float32).contiguous()
        b = norm.bias.detach().to(self.device, torch.float32).contiguous() if norm.bias is not None else None
        return (w, b, norm.eps, norm.kind)

    def _lm_head(self, head):
        from .quantization import QuantizedLinear

        if isinstance(head, QuantizedLinear):
            return head.dequantize().to(self.device, self.dtype).contiguous()
        return head.weight.detach().to(self.device, self.dtype).contiguous()

    def _experts(self, layer, moe) -> None:
        quant = getattr(moe, "quant", None)
        dev = self.device
        if quant is not None and self.native:
            layer.fmt = 2 if quant["bits"] == 4 else 1
            layer.group_in, layer.group_down = quant["group_in"], quant["group_down"]
            layer.q_gu, layer.s_gu = moe.q_gate_up.to(dev).contiguous(), moe.s_gate_up.to(dev).contiguous()
            layer.q_d, layer.s_d = moe.q_down.to(dev).contiguous(), moe.s_down.to(dev).contiguous()
            if layer.fmt == 1:  # int8 uses one scale per row: the layout already has groups == 1 when per-channel
                if layer.s_gu.size(-1) != 1 or layer.s_d.size(-1) != 1:
                    raise Unsupported("int8 decode kernels need per-channel (one group per row) scales")
        else:
            layer.fmt = 0
            layer.group_in = layer.group_down = 0
            wgu = torch.stack([moe.expert_weights(e)[0] for e in range(moe.num_local_experts)])
            wd = torch.stack([moe.expert_weights(e)[1] for e in range(moe.num_local_experts)])
            layer.q_gu, layer.s_gu = wgu.detach().to(dev, self.dtype).contiguous(), None
            layer.q_d, layer.s_d = wd.detach().to(dev, self.dtype).contiguous(), None

    # ---- the one-token step ------------------------------------------------------------------------
    def _embed(self, tokens: Tensor, positions: Tensor) -> Tensor:
        x = self.tok_emb[tokens]
        if self.learned:
            x = x + self.pos_emb[positions.long()]
        return x

    def _step(self, batch: int) -> Tensor:
        return self._step_native(batch) if self.native else self._step_torch(batch)

    def _step_torch(self, batch: int) -> Tensor:
        """fp32 PyTorch step (CPU oracle)."""
        from ..models.layers import apply_rope_reference, rope_tables, rms_norm_reference

        tokens, positions = self.tokens_in[:batch], self.positions_in[:batch]
        x = self._embed(tokens, positions).float()
        hq, hkv, d = self.heads, self.kv_heads, self.head_dim
        pos = positions.long()
        for layer in self.layers:
            n1 = self._apply_norm(x, layer.norm1)
            qkv = F.linear(n1, layer.wqkv.float(), layer.bqkv)
            q = qkv[:, : hq * d].view(batch, 1, hq, d)
            k = qkv[:, hq * d:(hq + hkv) * d].view(batch, 1, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(batch, hkv, d)
            if not self.learned:
                cos, sin = self.cos[pos], self.sin[pos]
                q = torch.stack([apply_rope_reference(q[i:i + 1], cos[i:i + 1], sin[i:i + 1]) for i in range(batch)]).view(batch, 1, hq, d)
                k = torch.stack([apply_rope_reference(k[i:i + 1], cos[i:i + 1], sin[i:i + 1]) for i in range(batch)]).view(batch, 1, hkv, d)
            for i in range(batch):
                layer.keys[i, :, pos[i]] = k[i, 0].to(layer.keys.dtype)
                layer.values[i, :, pos[i]] = v[i].to(layer.values.dtype)
            keys = layer.keys[:batch].float().repeat_interleave(hq // hkv, dim=1)
            values = layer.values[:batch].float().repeat_interleave(hq // hkv, dim=1)
            visible = (torch.arange(self.capacity, device=x.device)[None, :] <= pos[:, None]).view(batch, 1, 1, -1)
            att = F.scaled_dot_product_attention(q.transpose(1, 2), keys, values, attn_mask=visible)
            x = x + F.linear(att.reshape(batch, hq * d), layer.wo.float(), layer.bo)
            n2 = self._apply_norm(x, layer.norm2)
            scores = F.linear(n2, layer.router) / layer.temperature
            probs = scores.softmax(-1)
            chosen = (scores + layer.bias if layer.bias is not None else probs).topk(layer.top_k, dim=-1).indices
            weights = probs.gather(1, chosen)
            weights = weights / weights.sum(-1, keepdim=True)
            f = layer.ffn
            if self.ep is not None:  # this rank's experts only; the group's partial outputs are summed below
                local = layer.q_gu.size(0)
                first = self.ep.rank * local
                mine = (chosen >= first) & (chosen < first + local)
                weights = weights * mine
                chosen = (chosen - first).clamp(0, local - 1)
            wgu = layer.q_gu[chosen].float()          # [B, k, 2F, H]
            wd = layer.q_d[chosen].float()            # [B, k, H, F]
            g = torch.einsum("bkfh,bh->bkf", wgu[:, :, :f], n2)
            u = torch.einsum("bkfh,bh->bkf", wgu[:, :, f:], n2)
            out = torch.einsum("bkhf,bkf->bkh", wd, F.silu(g) * u)
            moe_out = (out * weights[..., None]).sum(1)
            if self.ep is not None:
                import torch.distributed as dist

                dist.all_reduce(moe_out, group=self.ep.group)
            x = x + moe_out
        del rope_tables, rms_norm_reference
        x = self._apply_norm(x, self.final_norm)
        return F.linear(x, self.lm_head.float())

    @staticmethod
    def _apply_norm(x: Tensor, norm) -> Tensor:
        w, b, eps, kind = norm
        if kind == "layernorm":
            return F.layer_norm(x.float(), (x.size(-1),), w, b, eps)
        xf = x.float()
        return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w

    def _native_norm(self, x: Tensor, norm) -> Tensor:
        C = self._C
        w, b, eps, kind = norm
        y = torch.empty_like(x)
        rstd = torch.empty(x.size(0), device=x.device)
        mean = None if kind == "rmsnorm" else torch.empty(x.size(0), device=x.device)
        C.norm_fwd(x, None, None, w, b, y, mean, rstd, eps, kind == "rmsnorm")
        return y

    def _step_native(self, batch: int) -> Tensor:
        """One decode step on the native kernels: 8 launches per layer, all with programmatic dependent launch.

        combine(previous MoE output) + norm1 -> QKV GEMV (+bias) -> split-K attention with RoPE and the cache append
        of the new token folded in (chunk merge in the same launch) -> out-proj GEMV (+bias +residual) -> norm2 ->
        routing (logits + top-k + lists) -> SwiGLU grouped GEMV over the routed experts -> down grouped GEMV. The
        last layer's MoE output is combined inside the final norm."""
        from ..ops import ext

        C = self._C = ext()
        dev = self.tok_emb.device
        tokens, positions = self.tokens_in[:batch], self.positions_in[:batch]
        hq, hkv, d, H = self.heads, self.kv_heads, self.head_dim, self.hidden
        bf = torch.bfloat16
        chunks = C.decode_attn_chunks(self.capacity)
        tickets = self._tickets
        x = None
        pending = None  # (y, slot, top_w, k) of the previous layer's MoE, or its layer index (expert-parallel)
        if self.ep is not None:
            C.ep_decode_tick(self._ep_step)  # a fresh exchange target for this step (also on every graph replay)
        for li, layer in enumerate(self.layers):
            w1, b1, eps1, kind1 = layer.norm1
            n1 = torch.empty(batch, H, device=dev, dtype=bf)
            if x is None:  # embedding (+ learned position) fused into the first norm
                x = torch.empty(batch, H, device=dev, dtype=bf)
                C.decode_combine_norm(None, tokens, self.tok_emb, self.pos_emb if self.learned else None, positions,
                                      None, None, None, 0, w1, b1, eps1, kind1 == "rmsnorm", x, n1)
            else:
                x_res = torch.empty_like(x)
                self._combine_norm(x, pending, layer.norm1, x_res, n1)
                x = x_res
            qkv = torch.empty(batch, (hq + 2 * hkv) * d, device=dev, dtype=bf)
            C.grouped_gemv(n1, layer.wqkv, None, qkv.size(1), H, 0, 0, False, None, None, None, 1, batch,
                           qkv, False, layer.bqkv, None, None)
            part_o = torch.empty(batch * hq * chunks * d, device=dev, dtype=torch.float32)
            part_ml = torch.empty(batch * hq * chunks * 2, device=dev, dtype=torch.float32)
            att = torch.empty(batch, hq * d, device=dev, dtype=bf)
            # RoPE and the cache append of the new token happen inside the attention launch
            C.decode_attention_rope(qkv, positions, self.cos, self.sin, not self.learned, layer.keys[:batch],
                                    layer.values[:batch], hq, 1.0 / math.sqrt(d), part_o, part_ml, tickets, att)
            x_new = torch.empty_like(x)  # out-projection with bias and the residual add in the GEMV epilogue
            C.grouped_gemv(att, layer.wo, None, H, hq * d, 0, 0, False, None, None, None, 1, batch, x_new,
                           False, layer.bo, x, None)
            x = x_new
            w2, b2, eps2, kind2 = layer.norm2
            n2 = torch.empty_like(x)
            C.decode_combine_norm(x, None, None, None, None, None, None, None, 0, w2, b2, eps2, kind2 == "rmsnorm",
                                  None, n2)
            pending = self._moe_native(layer, n2, batch, li)
        xf = torch.empty_like(x)
        self._combine_norm(x, pending, self.final_norm, None, xf)
        logits = torch.empty(batch, self.vocab, device=dev, dtype=bf)
        C.grouped_gemv(xf, self.lm_head, None, self.vocab, H, 0, 0, False, None, None, None, 1, batch, logits,
                       False, None, None, None)
        return logits.float()

    def _combine_norm(self, x: Tensor, pending, norm, x_out: Optional[Tensor], n_out: Tensor) -> None:
        """x (+ the previous layer's MoE output) -> (x_out, norm(x_out)). Single GPU: weighted rows of the routed
        expert outputs; expert-parallel: every rank's partial outputs from the exchange planes, in rank order."""
        w, b, eps, kind = norm
        if self.ep is not None:
            self._C.decode_combine_norm_parts(x, self._ep_parts, self._ep_step, pending, len(self.layers),
                                              self._ep_world, self.max_batch, w, b, eps, kind == "rmsnorm", x_out,
                                              n_out)
            return
        y, slot, top_w, k = pending
        self._C.decode_combine_norm(x, None, None, None, None, y, slot, top_w, k, w, b, eps, kind == "rmsnorm", x_out,
                                    n_out)

    def _moe_native(self, layer, n2: Tensor, batch: int, index: int = 0):
        """Fused decode routing (no capacity) -> grouped dequant SwiGLU GEMV -> grouped down GEMV.

        Returns (y [routes, H] route-major, route_slot, top_w, k); the combine happens in the next norm. Expert-parallel:
        only this rank's experts run (the other routes' rows stay zero), the per-token partial outputs are pushed into
        every rank's exchange plane and the wait for all peers' planes follows; returns the layer index."""
        C = self._C
        dev = n2.device
        E, k, f = layer.num_experts, layer.top_k, layer.ffn
        routes = batch * k
        cnt = torch.empty(E, device=dev, dtype=torch.int32)
        off = torch.empty(E, device=dev, dtype=torch.int32)
        order = torch.empty(routes, device=dev, dtype=torch.int32)
        slot = torch.empty(routes, device=dev, dtype=torch.int32)
        top_w = torch.empty(batch, k, device=dev, dtype=torch.float32)
        logits = torch.empty(batch, E, device=dev, dtype=torch.float32)
        active = torch.empty(min(E, routes), device=dev, dtype=torch.int32)
        first, groups = 0, E
        if self.ep is not None:
            first, groups = self._ep_first, self._ep_local
            C.decode_route_local(n2, layer.router, layer.bias, k, layer.temperature, logits, cnt, off, order, slot,
                                 top_w, active, self._tickets, first, groups)
        else:
            C.decode_route(n2, layer.router, layer.bias, k, layer.temperature, logits, cnt, off, order, slot, top_w,
                           active, self._tickets)
        cnt_l, off_l = cnt[first:first + groups], off[first:first + groups]
        h = torch.empty(routes, f, device=dev, dtype=torch.bfloat16)
        C.grouped_gemv(n2, layer.q_gu, layer.s_gu, f, self.hidden, layer.group_in, layer.fmt, True, order, off_l,
                       cnt_l, groups, 0, h, True, None, None, active)
        alloc = torch.zeros if self.ep is not None else torch.empty  # routes to other ranks' experts add zero
        y = alloc(routes, self.hidden, device=dev, dtype=torch.bfloat16)
        C.grouped_gemv(h, layer.q_d, layer.s_d, self.hidden, f, layer.group_down, layer.fmt, False, None, off_l,
                       cnt_l, groups, 0, y, True, None, None, active)
        if self.ep is None:
            return y, slot, top_w, k
        layers = len(self.layers)
        C.ep_decode_push(y, slot, top_w, k, self.max_batch, self._ep_peers, self._ep_plane, index, layers,
                         self._ep_me, self._ep_peer_flags, self._ep_step, self._ep_done)
        C.ep_decode_wait(self._ep_flags, self._ep_world, self._ep_step, index, layers, self._ep_timeout)
        return index

    # ---- graphs ------------------------------------------------------------------------------------
    @torch.no_grad()
    def _capture(self) -> None:
        batch = self.max_batch
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
                self.logits[:batch].copy_(self._step(batch))
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.logits[:batch].copy_(self._step(batch))
        self.graph = graph
        for layer in self.layers:
            layer.keys.zero_()
            layer.values.zero_()

    @property
    def uses_graph(self) -> bool:
        return self.graph is not None

    @property
    def description(self) -> str:
        base = "KV cache" if not self.native else "KV cache + native sm_100a kernels"
        return base + (" + CUDA graph" if self.graph is not None else "")

    # ---- prefill -------------------------------------------------------------------------------------
    @torch.no_grad()
    def _prefill(self, prompts: Tensor, first_row: int = 0) -> None:
        """Read ``prompts [B, n]`` in one pass (no expert capacity) and leave their keys/values in cache rows
        ``first_row .. first_row + B - 1`` (a continuous batcher fills one slot at a time)."""
        batch, n = prompts.shape
        self.length = n
        if n == 0:
            return
        rows = slice(first_row, first_row + batch)
        model = self.model
        saved = [(moe.capacity_factor, moe.drop_overflow_tokens, moe.kernel) for moe in model.moes()]
        for moe in model.moes():
            moe.drop_overflow_tokens = False
            if self.ep is not None:
                moe.kernel = "loop"  # expert-parallel prefill: the per-expert exchange path (fp32, any device)
        try:
            hidden = model.embed(prompts.to(self.device))
            hq, hkv, d = self.heads, self.kv_heads, self.head_dim
            for block, layer in zip(model.blocks, self.layers):
                att = block.attention
                normed = block.attention_norm(hidden)
                q, k, v = att.qkv(normed) if not self.native else self._native_qkv(att, normed, batch, n)
                layer.keys[rows, :, :n] = k.transpose(1, 2).to(layer.keys.dtype)
                layer.values[rows, :, :n] = v.transpose(1, 2).to(layer.values.dtype)
                if self.native:
                    o = self._native_attention(q, k, v, batch, n)
                    from ..ops.linear import linear

                    hidden = linear(o.reshape(-1, hq * d), att.out_proj.weight, att.out_proj.bias,
                                    hidden.reshape(-1, self.hidden)).view(batch, n, self.hidden)
                else:
                    if hkv != hq:
                        k = k.repeat_interleave(hq // hkv, dim=2)
                        v = v.repeat_interleave(hq // hkv, dim=2)
                    o = F.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                                       v.transpose(1, 2).float(), is_causal=True)
                    o = o.transpose(1, 2).reshape(batch, n, hq * d).to(hidden.dtype)
                    hidden = hidden + att.out_proj(o)
                moe_out = block.moe(block.moe_norm(hidden))[0]
                hidden = hidden + moe_out
        finally:
            for moe, (cf, drop, kernel) in zip(model.moes(), saved):
                moe.capacity_factor, moe.drop_overflow_tokens, moe.kernel = cf, drop, kernel

    def _native_attention(self, q: Tensor, k: Tensor, v: Tensor, batch: int, n: int) -> Tensor:
        """Causal flash attention over the (already rotated) prompt; q/k/v are views into the packed QKV rows."""
        hq, hkv, d = self.heads, self.kv_heads, self.head_dim
        qkv = self._qkv_rows
        o = torch.empty(batch * n, hq * d, device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty(batch, hq, n, device=qkv.device, dtype=torch.float32)
        self._C.flash_attn_fwd(qkv[:, : hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:], o, lse,
                               batch, n, hq, hkv, d, 1.0 / math.sqrt(d))
        return o

    def _native_qkv(self, att, normed: Tensor, batch: int, n: int):
        from ..ops.linear import linear

        hq, hkv, d = self.heads, self.kv_heads, self.head_dim
        qkv = linear(normed.reshape(-1, self.hidden), att.in_proj_weight, att.in_proj_bias).contiguous()
        if not self.learned:
            from ..ops.attention import rope_cache

            cos, sin = rope_cache(n, d, self.config.rope_theta, qkv.device)
            self._C.rope_apply(qkv, hq + hkv, d, n, None, cos, sin, False)
        self._qkv_rows = qkv
        qkv = qkv.view(batch, n, hq + 2 * hkv, d)
        return qkv[:, :, :hq], qkv[:, :, hq:hq + hkv], qkv[:, :, hq + hkv:]

    # ---- batched generation ------------------------------------------------------------------------------
    @torch.no_grad()
    def run_step(self, tokens: Tensor, positions: Tensor) -> Tensor:
        """One step for ``tokens [B]`` at ``positions [B]``; returns fp32 logits ``[B, V]`` (a reused buffer)."""
        batch = tokens.numel()
        self.tokens_in[:batch].copy_(tokens)
        self.positions_in[:batch].copy_(positions.to(torch.int32))
        if self.graph is not None and batch == self.max_batch:
            self.graph.replay()
        else:
            self.logits[:batch].copy_(self._step(batch))
        return self.logits[:batch]

    @torch.no_grad()
    def generate(self, prompts: Tensor, max_new: int) -> Tensor:
        """Greedy decoding of ``prompts [B, P]`` (equal lengths) for ``max_new`` tokens; returns ``[B, max_new]``."""
        if self.native and not hasattr(self, "_C"):
            from ..ops import ext

            self._C = ext()
        batch, plen = prompts.shape
        if plen + max_new > self.capacity:
            raise ValueError(f"prompt + new tokens ({plen + max_new}) exceed the context {self.capacity}")
        prompts = prompts.to(self.device)
        self._prefill(prompts[:, :-1])
        out = torch.empty(batch, max_new, dtype=torch.long, device=self.device)
        token = prompts[:, -1]
        for i in range(max_new):
            positions = torch.full((batch,), plen - 1 + i, dtype=torch.int32, device=self.device)
            logits = self.run_step(token, positions)
            token = logits.argmax(-1)
            out[:, i] = token
        return out

    # ---- batch-1 interface (reference parity) ----------------------------------------------------------
    def reset(self) -> None:
        self.length = 0
        self.tokens = []

    @torch.no_grad()
    def _run(self, token: int) -> None:
        t = torch.tensor([token], device=self.device)
        p = torch.tensor([self.length], dtype=torch.int32, device=self.device)
        self.run_step(t, p)
        self.length += 1
        self.tokens.append(token)

    def feed(self, ids: list) -> Tensor:
        window = list(ids)[-self.capacity:]
        if not window:
            raise ValueError("nothing to decode from")
        if self.native and not hasattr(self, "_C"):
            from ..ops import ext

            self._C = ext()
        self.reset()
        self._prefill(torch.tensor([window[:-1]], device=self.device))
        self.tokens = list(window[:-1])
        self._run(window[-1])
        return self.logits[0]

    def append(self, token: int) -> Tensor:
        if self.length >= self.capacity:
            keep = self.tokens[-(self.capacity // 2):]
            self.reset()
            self._prefill(torch.tensor([keep], device=self.device))
            self.tokens = list(keep)
        self._run(token)
        return self.logits[0]

    def warm(self, temperature: float, top_k: int = 0, top_p: float = 1.0, duration: int = 64) -> None:
        for _ in self.stream([0, 0], duration, temperature=temperature, top_k=top_k, top_p=top_p):
            pass
        self.reset()

    @torch.no_grad()
    def stream(self, ids: list, max_new: int, *, temperature: float, top_k: int = 0, top_p: float = 1.0,
               valid_ids: Optional[int] = None, unk_id: Optional[int] = None,
               generator: Optional[torch.Generator] = None) -> Iterator[int]:
        """Read ``ids`` and yield up to ``max_new`` sampled tokens (greedy when ``temperature <= 0``)."""
        if not ids:
            raise ValueError("nothing to decode from")
        mask = torch.zeros(self.vocab, device=self.device)
        if valid_ids is not None and valid_ids < self.vocab:
            mask[valid_ids:] = float("-inf")
        if unk_id is not None and 0 <= unk_id < self.vocab:
            mask[unk_id] = float("-inf")
        logits = self.feed(ids)
        produced = 0
        while produced < max_new:
            row = logits + mask
            if temperature <= 0:
                token = int(row.argmax())
            else:
                noise = torch.rand(self.vocab, generator=generator, device=generator.device if generator is not None
                                   else self.device).to(self.device).clamp(1e-20, 1.0 - 1e-7)
                token = int((filter_logits(row / temperature, top_k, top_p) - torch.log(-torch.log(noise))).argmax())
            yield token
            produced += 1
            if produced >= max_new:
                return
            logits = self.append(token)


@contextlib.contextmanager
def capture_mode():
    with torch.inference_mode(False), torch.no_grad():
        yield
