"""Decoder-only sparse-MoE causal language model.

Behaviour follows the reference ``QuantaWeaveBlock`` / ``QuantaWeaveMoEForCausalLM``
(``src/quantweave_moe_model.py:275-460``): pre-norm blocks ``h += Attn(Norm(h))``, ``h += MoE(Norm(h))``; token
embedding (+ learned positions on the first pipeline stage); final norm + ``lm_head`` on the last stage; loss
``CE(logits[:, :-1], labels[:, 1:]) + aux_coef * mean(aux) + domain_coef * domain``; runtime controls
``set_routing_controls``, ``set_collect_stats``, ``set_moe_kernel``, ``set_static_dispatch``, ``routing_stats``.

On CUDA the head and loss run through a fused chunked linear-cross-entropy kernel so full-vocabulary logits are
never materialised during training (``return_logits=False``).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from ..config import QuantaWeaveConfig
from .layers import Attention, Norm
from .moe import TopKMoE


class QuantaWeaveBlock(nn.Module):
    def __init__(self, config: QuantaWeaveConfig, expert_parallel=None) -> None:
        super().__init__()
        tp_size = getattr(expert_parallel, "tp_size", 1)
        tp_rank = getattr(expert_parallel, "tp_rank", 0)
        self.attention_norm = Norm(config.hidden_size, config.norm_type, config.norm_eps)
        if tp_size > 1:
            from ..parallel.tensor_parallel import TensorParallelAttention

            self.attention = TensorParallelAttention(config, expert_parallel)
        else:
            self.attention = Attention(config)
        self.moe_norm = Norm(config.hidden_size, config.norm_type, config.norm_eps)
        if expert_parallel is None:
            self.moe = TopKMoE(config)
        else:
            from ..parallel.expert_parallel import ExpertParallelMoE

            self.moe = ExpertParallelMoE(config, expert_parallel)
        del tp_rank

    def forward(self, hidden: Tensor, causal_mask: Optional[Tensor] = None, token_domains: Optional[Tensor] = None,
                num_domains: int = 0):
        """``causal_mask`` keeps the reference's argument order (``src/quantweave_moe_model.py:293``); attention here
        is always causal, so the mask itself is not needed."""
        del causal_mask
        if hidden.is_cuda and type(self.attention) is Attention:
            from ..ops.attention import self_attention

            # residual add fused into the output-projection GEMM epilogue
            hidden = self_attention(self.attention, self.attention_norm(hidden), residual=hidden)
        else:
            hidden = hidden + self.attention(self.attention_norm(hidden))
        moe_out, balance, dropped, overflow, domain = self.moe(self.moe_norm(hidden), token_domains, num_domains)
        return hidden + moe_out, balance, dropped, overflow, domain


class QuantaWeaveMoEForCausalLM(nn.Module):
    def __init__(self, config: QuantaWeaveConfig, expert_parallel=None, pipeline=None) -> None:
        super().__init__()
        if expert_parallel is not None and pipeline is not None and getattr(expert_parallel, "world_size", 1) > 1:
            raise ValueError("pipeline parallelism cannot be combined with expert/tensor parallelism")
        self.config = config
        self.expert_parallel = expert_parallel
        self.pipeline = pipeline
        first = pipeline is None or pipeline.stage == 0
        last = pipeline is None or pipeline.stage == pipeline.num_stages - 1
        layer_count = config.layers if pipeline is None else pipeline.layer_end - pipeline.layer_start
        self.router_aux_loss_coef = config.router_aux_loss_coef
        self.domain_specialization_coef = 0.0
        self.activation_checkpointing = False
        self.token_embedding = nn.Embedding(config.vocab_size, config.hidden_size) if first else None
        learned = config.position_embedding == "learned"
        self.position_embedding = nn.Embedding(config.max_sequence_length, config.hidden_size) if (first and learned) else None
        self.blocks = nn.ModuleList(QuantaWeaveBlock(config, expert_parallel) for _ in range(layer_count))
        self.final_norm = Norm(config.hidden_size, config.norm_type, config.norm_eps) if last else None
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False) if last else None
        if config.init_std is not None:
            with torch.no_grad():
                for emb in (self.token_embedding, self.position_embedding):
                    if emb is not None:
                        emb.weight.normal_(0.0, config.init_std)
                if self.lm_head is not None:
                    self.lm_head.weight.normal_(0.0, config.init_std)

    # ---- runtime controls ----------------------------------------------------
    def moes(self) -> list[TopKMoE]:
        return [block.moe for block in self.blocks]

    def set_routing_controls(self, capacity_factor: Optional[float] = None, drop_overflow_tokens: Optional[bool] = None,
                             overflow_policy: Optional[str] = None, router_temperature: Optional[float] = None,
                             router_aux_loss_coef: Optional[float] = None) -> None:
        if overflow_policy is not None and overflow_policy not in {"drop", "residual"}:
            raise ValueError("overflow_policy must be 'drop' or 'residual'")
        if router_temperature is not None and router_temperature <= 0:
            raise ValueError("router_temperature must be positive")
        if capacity_factor is not None and capacity_factor < 0:
            raise ValueError("capacity_factor must be >= 0")
        updates = {"capacity_factor": capacity_factor, "drop_overflow_tokens": drop_overflow_tokens,
                   "overflow_policy": overflow_policy, "router_temperature": router_temperature}
        for name, value in updates.items():
            if value is None:
                continue
            for moe in self.moes():
                setattr(moe, name, value)
            setattr(self.config, name, value)
        if router_aux_loss_coef is not None:
            self.router_aux_loss_coef = router_aux_loss_coef
            self.config.router_aux_loss_coef = router_aux_loss_coef

    def set_collect_stats(self, enabled: bool) -> None:
        for moe in self.moes():
            moe.collect_stats = enabled

    def set_moe_kernel(self, kernel: str) -> str:
        """Expert compute path: ``loop`` (per-expert oracle), ``native``/``triton`` (grouped tcgen05 kernels; the
        reference's ``triton`` name is accepted as an alias) or ``auto``. Returns the active path."""
        if kernel not in {"loop", "triton", "native", "auto"}:
            raise ValueError("kernel must be loop, native (alias triton) or auto")
        device = next(self.parameters()).device
        from ..ops import native_available

        available = device.type == "cuda" and native_available()
        if kernel in {"triton", "native"} and not available:
            raise RuntimeError("the native MoE kernels need a CUDA device and the compiled quantaweave_b200._C extension")
        active = "native" if (kernel in {"triton", "native"} or (kernel == "auto" and available)) else "loop"
        for moe in self.moes():
            moe.kernel = active
        return active

    def set_static_dispatch(self, enabled: bool) -> None:
        for moe in self.moes():
            moe.static_dispatch = enabled

    def routing_stats(self) -> list[dict[str, Tensor]]:
        return [moe.last_stats for moe in self.moes()]

    def parameter_parts(self) -> list:
        """``(module, parameters)`` pairs in the order the forward first uses the parameters: the model itself
        (embeddings, and every parameter not listed later), each block, then the final norm (final norm and LM
        head, unless tied to the embedding). An optimizer that overlaps its update with the next forward waits for a
        part's update in a forward pre-hook on that part's module."""
        first = {id(p) for m in (self.token_embedding, self.position_embedding) if m is not None
                 for p in m.parameters()}
        blocks = [(b, [p for p in b.parameters() if id(p) not in first]) for b in self.blocks]
        taken = set(first) | {id(p) for _, ps in blocks for p in ps}
        final = [] if self.final_norm is None else [
            p for m in (self.final_norm, self.lm_head) if m is not None for p in m.parameters() if id(p) not in taken]
        taken |= {id(p) for p in final}
        head = [p for p in self.parameters() if id(p) not in taken or id(p) in first]
        parts = [(self, head)] + blocks
        if self.final_norm is not None:
            parts.append((self.final_norm, final))
        return parts

    # ---- forward ---------------------------------------------------------------
    def embed(self, input_ids: Tensor) -> Tensor:
        _, sequence = input_ids.shape
        if self.position_embedding is not None:
            if sequence > self.config.max_sequence_length:
                raise ValueError("input sequence exceeds max_sequence_length")
            positions = torch.arange(sequence, device=input_ids.device)
            return self.token_embedding(input_ids) + self.position_embedding(positions)[None, :, :]
        return self.token_embedding(input_ids)

    def run_blocks(self, hidden: Tensor, token_domains: Optional[Tensor] = None, num_domains: int = 0):
        balance, dropped, overflow, domain = [], [], [], []
        for block in self.blocks:
            if self.activation_checkpointing and self.training:
                hidden, b, d, o, dom = checkpoint(block, hidden, None, token_domains, num_domains, use_reentrant=False)
            else:
                hidden, b, d, o, dom = block(hidden, None, token_domains, num_domains)
            balance.append(b)
            dropped.append(d)
            overflow.append(o)
            domain.append(dom)
        return hidden, balance, dropped, overflow, domain

    def head(self, hidden: Tensor) -> Tensor:
        return self.lm_head(self.final_norm(hidden))

    def lm_loss(self, hidden: Tensor, labels: Tensor) -> Tensor:
        """Mean next-token cross-entropy of ``lm_head(final_norm(hidden))[:, :-1]`` against ``labels[:, 1:]``."""
        normed = self.final_norm(hidden)
        if normed.is_cuda:
            from ..ops import cross_entropy as ce_ops

            # every position is scored against the next token; the last one has none (ignore index)
            shifted = torch.cat([labels[:, 1:], labels.new_full((labels.size(0), 1), ce_ops.IGNORE_INDEX)], dim=1)
            return ce_ops.linear_cross_entropy(normed, self.lm_head.weight, shifted)
        logits = self.lm_head(normed)
        return F.cross_entropy(logits[:, :-1].reshape(-1, logits.size(-1)), labels[:, 1:].reshape(-1))

    # ---- sequence parallelism (attention TP and expert EP over the same ranks) ------------------------------
    def _sequence_parallel(self):
        ep = self.expert_parallel
        return ep if ep is not None and getattr(ep, "sequence_parallel", False) else None

    def _shard_rows(self, hidden: Tensor, token_domains: Optional[Tensor], ctx):
        """Keep this rank's contiguous share of the flattened ``batch x sequence`` rows (as a [1, rows, H] batch)."""
        batch, seq, width = hidden.shape
        total = batch * seq
        if total % ctx.world_size:
            raise ValueError(f"batch x sequence ({total}) must be divisible by the sequence-parallel size "
                             f"{ctx.world_size}")
        rows = total // ctx.world_size
        start = ctx.rank * rows
        for block in self.blocks:
            block.attention.sp_shape = (batch, seq)
        local = hidden.reshape(total, width)[start:start + rows].reshape(1, rows, width)
        if token_domains is not None:
            token_domains = token_domains[start:start + rows]
        return local, token_domains, (start, rows)

    def _sequence_parallel_loss(self, hidden: Tensor, labels: Tensor, ctx, span: tuple) -> Tensor:
        """This rank's share of the batch-mean next-token CE, scaled so the mean over ranks is the batch mean:
        ``world * (sum of CE over this rank's rows) / (valid positions in the whole batch)``."""
        from ..ops import cross_entropy as ce_ops

        start, rows = span
        ignore = ce_ops.IGNORE_INDEX
        shifted = torch.cat([labels[:, 1:], labels.new_full((labels.size(0), 1), ignore)], dim=1).reshape(-1)
        local = shifted[start:start + rows]
        total_valid = (shifted != ignore).sum().clamp(min=1)
        normed = self.final_norm(hidden)
        if normed.is_cuda:
            mean = ce_ops.linear_cross_entropy(normed, self.lm_head.weight, local.view(1, rows))
            ce_sum = mean * (local != ignore).sum()
        else:
            logits = self.lm_head(normed).reshape(rows, -1)
            ce_sum = F.cross_entropy(logits.float(), local, ignore_index=ignore, reduction="sum")
        return ce_sum * ctx.world_size / total_valid

    def forward(self, input_ids: Tensor, labels: Optional[Tensor] = None, domain_ids: Optional[Tensor] = None,
                num_domains: int = 0, return_logits: bool = True) -> dict:
        """With sequence parallelism every rank gets the same ``input_ids``; it keeps its share of the token rows
        through the blocks, ``logits`` are this rank's rows (``[1, rows, vocab]``) and ``loss`` is this rank's
        share scaled so that the mean over ranks is the batch loss."""
        if self.pipeline is not None and getattr(self.pipeline, "num_stages", 1) > 1:
            raise RuntimeError("a pipeline-stage model holds only some layers; drive it with PipelineEngine")
        hidden = self.embed(input_ids)
        token_domains = None
        if domain_ids is not None and self.domain_specialization_coef != 0 and num_domains > 1:
            token_domains = domain_ids.repeat_interleave(input_ids.size(1))
        sp = self._sequence_parallel()
        if sp is not None:
            hidden, token_domains, span = self._shard_rows(hidden, token_domains, sp)
        hidden, balance, dropped, overflow, domain = self.run_blocks(hidden, token_domains, num_domains)
        result: dict = {
            "router_aux_loss": torch.stack(balance).mean(),
            "domain_loss": torch.stack(domain).mean(),
            "expert_indices": [moe.last_top_indices for moe in self.moes()],
            "dropped_routes": torch.stack(dropped).sum(),
            "overflow_routes": torch.stack(overflow).sum(),
        }
        if sp is not None:
            if return_logits or labels is None:
                result["logits"] = self.head(hidden)
            ce = self._sequence_parallel_loss(hidden, labels, sp, span) if labels is not None else None
        elif return_logits or labels is None or not hidden.is_cuda:
            logits = self.head(hidden)
            result["logits"] = logits
            if labels is not None:
                ce = F.cross_entropy(logits[:, :-1].reshape(-1, logits.size(-1)).float(), labels[:, 1:].reshape(-1))
        else:
            ce = self.lm_loss(hidden, labels) if labels is not None else None
        if labels is not None:
            result["loss"] = (ce + self.router_aux_loss_coef * result["router_aux_loss"]
                              + self.domain_specialization_coef * result["domain_loss"])
        return result
