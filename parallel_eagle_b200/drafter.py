"""The feature-conditioned parallel multi-token drafter (B200 build).

Same module tree, parameter names, initialisation order and checkpoint layout
as the reference ``ParallelDrafter`` (``src/pe/drafter.py:36-299``): a drafter
state dict saved by either implementation loads into the other.  The shared
frozen embedding, LM head and final norm are held in 1-tuples so they stay out
of ``parameters()`` and the checkpoint (reference ``drafter.py:78-83``).

Compute goes through libpe_b200: the generic ``forward(x, position_ids, bias)``
uses the autograd-enabled kernels of :mod:`parallel_eagle_b200.nn`; the training
step (:func:`parallel_eagle_b200.partition.mtp_backward`) runs the fused
forward/backward engine in :mod:`parallel_eagle_b200.engine`.
"""

from __future__ import annotations

from pathlib import Path

import torch
from torch import nn

from . import _lib as L
from . import ops
from .config import DrafterConfig
from .masks import mtp_allow_mask, mtp_labels, mtp_position_ids, to_additive_bias
from .nn import DecoderLayer, RMSNorm, build_rope_cache, linear, rms_norm


class ParallelDrafter(nn.Module):
    def __init__(
        self,
        *,
        hidden: int,
        n_heads: int,
        n_kv_heads: int,
        intermediate: int,
        vocab: int,
        feature_dim: int,
        rope_theta: float,
        eps: float,
        num_layers: int,
        max_depth: int,
        embed_module: nn.Module,
        lm_head_module: nn.Module,
        final_norm_module: nn.Module,
    ):
        super().__init__()
        self.hidden = hidden
        self.head_dim = hidden // n_heads
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.intermediate = intermediate
        self.rope_theta = rope_theta
        self.eps = eps
        self.max_depth = max_depth
        self.vocab = vocab
        self.feature_dim = feature_dim
        self.num_feature_layers = feature_dim // hidden
        # registration order matches the reference so seeded inits are identical
        self.feat_norm = RMSNorm(hidden, eps)
        self.feat_proj = nn.Linear(feature_dim, hidden, bias=False)
        self.in_proj = nn.Linear(2 * hidden, hidden, bias=False)
        self.mask_emb = nn.Parameter(torch.zeros(hidden))
        self.h_shared = nn.Parameter(torch.zeros(hidden))
        self.layers = nn.ModuleList(
            DecoderLayer(hidden, n_heads, n_kv_heads, intermediate, rope_theta, eps)
            for _ in range(num_layers)
        )
        nn.init.normal_(self.mask_emb, std=0.02)
        nn.init.normal_(self.h_shared, std=0.02)
        self._embed = (embed_module,)
        self._lm_head = (lm_head_module,)
        self._final_norm = (final_norm_module,)
        self.grad_checkpoint = False
        self._engine = None

    @classmethod
    def from_target(cls, target, dcfg: DrafterConfig) -> ParallelDrafter:
        """Dimensions from the target's config (reference ``drafter.py:89-107``)."""
        c = target.config
        return cls(
            hidden=target.hidden_size,
            n_heads=c.num_attention_heads,
            n_kv_heads=getattr(c, "num_key_value_heads", c.num_attention_heads),
            intermediate=c.intermediate_size,
            vocab=target.vocab_size,
            feature_dim=target.feature_dim,
            rope_theta=getattr(c, "rope_theta", 10000.0),
            eps=getattr(c, "rms_norm_eps", 1e-5),
            num_layers=dcfg.num_layers,
            max_depth=dcfg.max_depth,
            embed_module=target.get_input_embeddings(),
            lm_head_module=target.get_lm_head(),
            final_norm_module=target.get_final_norm(),
        )

    # ------------------------------------------------------------------ #
    @property
    def device(self) -> torch.device:
        return self.in_proj.weight.device

    @property
    def param_dtype(self) -> torch.dtype:
        return self.in_proj.weight.dtype

    def _embed_tokens(self, token_ids: torch.Tensor) -> torch.Tensor:
        return self._embed[0](token_ids)

    def lm_head(self, hidden: torch.Tensor) -> torch.Tensor:
        return self._lm_head[0](hidden)

    def frozen_heads(self):
        """``(embed [V,H], head [V,H], final-norm weight [H])``; they must already be
        in the parameter dtype on the parameter device, as in the reference, whose
        shared modules are not moved by ``.to()`` either."""
        e = self._embed[0].weight
        h = self._lm_head[0].weight
        n = self._final_norm[0].weight
        for name, t in (("embedding", e), ("LM head", h), ("final norm", n)):
            if t.device != self.device or t.dtype != self.param_dtype:
                raise ValueError(
                    f"shared {name} is {t.dtype} on {t.device} but the drafter is "
                    f"{self.param_dtype} on {self.device}; place the frozen target heads "
                    "with the drafter"
                )
        return e.detach(), h.detach(), n.detach()

    def real_input(self, token_ids: torch.Tensor, features: torch.Tensor) -> torch.Tensor:
        """``in_proj([emb(token); feat_proj(norm(feat))])`` (reference ``drafter.py:126-132``)."""
        L.require_cuda(token_ids, features)
        emb = self._embed_tokens(token_ids).to(self.param_dtype)
        f = features.to(self.param_dtype)
        f = self.feat_norm(f.unflatten(-1, (self.num_feature_layers, self.hidden)))
        feat = linear(f.flatten(-2), self.feat_proj.weight)
        return linear(torch.cat([emb, feat], dim=-1), self.in_proj.weight)

    def mask_input(self, n: int) -> torch.Tensor:
        """Shared prediction-slot input repeated ``n`` times (reference ``drafter.py:134-137``)."""
        cat = torch.cat([self.mask_emb, self.h_shared], dim=-1)[None]
        vec = linear(cat, self.in_proj.weight)[0]
        return vec.unsqueeze(0).expand(n, -1)

    def token_shared_input(self, token_ids: torch.Tensor) -> torch.Tensor:
        """``in_proj([emb(token); h_shared])`` for a drafted token whose target feature
        does not exist yet (reference ``drafter.py:139-145``)."""
        L.require_cuda(token_ids)
        emb = self._embed_tokens(token_ids).to(self.param_dtype)
        shared = self.h_shared.unsqueeze(0).expand(emb.shape[0], -1)
        return linear(torch.cat([emb, shared], dim=-1), self.in_proj.weight)

    @torch.no_grad()
    def draft_logits(self, context_ids: torch.Tensor, context_feats: torch.Tensor,
                     k: int) -> torch.Tensor:
        """Logits ``(k, V)`` for the ``k`` tokens following ``context_ids`` (reference
        ``drafter.py:195-236``).

        The packed sequence is the real context followed by ``k - 1`` prediction
        slots anchored at the last context position -- the partition layout with
        ``(a0, a1, K) = (p - 1, p, k)`` -- so the attention kernels re-derive the
        mask instead of reading a dense bias.  The frozen LM head runs on the ``k``
        prediction rows only: the last real slot (depth 0) and the prediction slots.
        """
        dev = self.device
        p = int(context_ids.shape[0])
        if p < 1 or k < 1:
            raise ValueError("draft_logits needs a non-empty context and k >= 1")
        m = p + (k - 1)
        x = torch.empty(m, self.hidden, dtype=self.param_dtype, device=dev)
        x[:p] = self.real_input(context_ids.to(dev), context_feats.to(dev))
        if k > 1:
            x[p:] = self.mask_input(k - 1)
        pos = torch.arange(m, device=dev)
        pos[p:] = (p - 1) + torch.arange(1, k, device=dev)
        layout = ops.AttnLayout(L.LAYOUT_PARTITION, a0=p - 1, a1=p, k=k)
        hidden = self.forward(x.unsqueeze(0), pos.unsqueeze(0), layout)[0]
        # depth 0 is predicted at the last real slot, depth d at slot p + d - 1
        return linear(hidden[p - 1 :], self._lm_head[0].weight)

    @torch.no_grad()
    def draft_logits_sequential(self, context_ids: torch.Tensor, context_feats: torch.Tensor,
                                k: int) -> torch.Tensor:
        """Greedy drafting by ``k`` causal forward passes, each appending the previous
        argmax token as :meth:`token_shared_input` (reference ``drafter.py:239-269``);
        the baseline parallel drafting replaces."""
        dev = self.device
        real_x = self.real_input(context_ids.to(dev), context_feats.to(dev))
        head = self._lm_head[0].weight
        drafted: list[int] = []
        out = []
        for _ in range(k):
            if drafted:
                tok = torch.tensor(drafted, device=dev)
                x = torch.cat([real_x, self.token_shared_input(tok)], dim=0)
            else:
                x = real_x
            s = x.shape[0]
            pos = torch.arange(s, device=dev).unsqueeze(0)
            causal = ops.AttnLayout(L.LAYOUT_PARTITION, a0=0, a1=s, k=1)
            hidden = self.forward(x.unsqueeze(0), pos, causal)[0]
            logits = linear(hidden[-1:], head)
            out.append(logits[0])
            # argmax with the first maximal column, as torch.argmax
            drafted.append(int(ops.topk_logprobs(logits, 1, raw=True)[1][0, 0]))
        return torch.stack(out)

    def forward(self, x: torch.Tensor, position_ids: torch.Tensor, bias) -> torch.Tensor:
        """``x`` (B, S, H), ``position_ids`` (B, S), ``bias`` (B|1, 1, S, S) additive
        (or an :class:`ops.AttnLayout`); returns final hidden states (B, S, H)
        (reference ``drafter.py:150-161``)."""
        L.require_cuda(x, position_ids)
        cos, sin = build_rope_cache(position_ids, self.head_dim, self.rope_theta)
        for layer in self.layers:
            x = layer(x, cos, sin, bias)
        fnorm = self._final_norm[0]
        return rms_norm(x, fnorm.weight, fnorm.eps)

    def build_training_packed(self, input_ids: torch.Tensor, features: torch.Tensor):
        """``(x, position_ids, bias, labels)`` of one example in the anchor-major
        layout (reference ``drafter.py:166-190``)."""
        k = self.max_depth
        n = input_ids.shape[0]
        dev = self.device
        s = n * k
        real_x = self.real_input(input_ids, features)
        x = torch.empty(s, self.hidden, dtype=self.param_dtype, device=dev)
        x[0::k] = real_x
        if k > 1:
            vec = self.mask_input(1)[0]
            for d in range(1, k):
                x[d::k] = vec
        position_ids = mtp_position_ids(n, k, device=dev).unsqueeze(0)
        bias = to_additive_bias(mtp_allow_mask(n, k, device=dev), self.param_dtype)
        labels = mtp_labels(input_ids, k)
        return x.unsqueeze(0), position_ids, bias, labels

    # ------------------------------------------------------------------ #
    def trainable_parameters(self):
        return [p for p in self.parameters() if p.requires_grad]

    def save_checkpoint(self, path, *, target_name: str) -> None:
        """Reference layout ``{state_dict, num_layers, max_depth, target_name}``
        (``drafter.py:277-286``); tensors are saved as standalone copies."""
        sd = {k: v.detach().clone() for k, v in self.state_dict().items()}
        torch.save(
            {"state_dict": sd, "num_layers": len(self.layers), "max_depth": self.max_depth,
             "target_name": target_name},
            path,
        )


def load_drafter(path, target) -> ParallelDrafter:
    """Rebuild a drafter from a checkpoint, re-sharing ``target``'s frozen heads
    (reference ``drafter.py:289-299``)."""
    if not Path(path).exists():
        raise FileNotFoundError(
            f"No drafter checkpoint at {path}. Train one first with `python -m pe.train`."
        )
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    dcfg = DrafterConfig(num_layers=ckpt["num_layers"], max_depth=ckpt["max_depth"])
    model = ParallelDrafter.from_target(target, dcfg)
    model.load_state_dict(ckpt["state_dict"])
    return model
