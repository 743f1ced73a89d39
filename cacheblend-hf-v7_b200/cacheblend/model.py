"""LayerwiseModel: an HF causal LM exposed layer by layer, with pre-RoPE K
capture through k_proj forward hooks (API of cacheblend-hf-v7 ``model.py``).

The seven public methods, the ``_pre_rope_k`` capture dict, the hook
installation and the ``__new__`` + field-assignment construction used by the
reference's runners are kept.  The class works with the installed
transformers (5.x): decoder layers are called with ``past_key_values`` and may
return a tensor or a tuple.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

_DTYPE_MAP = {"float16": torch.float16, "fp16": torch.float16,
              "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
              "float32": torch.float32, "fp32": torch.float32}


@dataclass
class LayerwiseOutput:
    """Prefill result: logits plus the full-length cache (HF DynamicCache)."""
    logits: torch.Tensor
    past_key_values: Optional[object] = None


def new_dynamic_cache():
    from transformers.cache_utils import DynamicCache
    return DynamicCache()


def attach_cache_layers(cache, kv: list[tuple[torch.Tensor, torch.Tensor]]):
    """Put per-layer (K, V) tensors of shape (1, Hkv, S, D) into a DynamicCache
    without copying them (DynamicCache.update would torch.cat a fresh copy)."""
    if hasattr(cache, "layers"):
        from transformers.cache_utils import DynamicLayer
        layers = []
        for k, v in kv:
            layer = DynamicLayer()
            layer.lazy_initialization(k, v)
            layer.keys, layer.values = k, v
            layers.append(layer)
        cache.layers = layers
    else:   # transformers 4.x: key_cache / value_cache lists
        cache.key_cache = [k for k, _ in kv]
        cache.value_cache = [v for _, v in kv]
    return cache


def _stack_linear(mods) -> Optional[torch.Tensor]:
    """One weight for bias-free nn.Linear modules that share an input size: each
    module's rows in order.  The modules' weights become row views of it (same
    values, one copy).  None if a module is not a bias-free nn.Linear or the
    weights differ in input size, dtype or device."""
    if any(not isinstance(m, torch.nn.Linear) or m.bias is not None for m in mods):
        return None
    ws = [m.weight for m in mods]
    if len({(w.shape[1], w.dtype, w.device) for w in ws}) != 1:
        return None
    stacked = torch.cat([w.detach() for w in ws], 0)
    off = 0
    for m in mods:
        n = m.weight.shape[0]
        m.weight.data = stacked[off:off + n]
        off += n
    return stacked


class LayerwiseModel:
    """HF causal LM wrapper with layer-by-layer forward and pre-RoPE K hooks."""

    def __init__(self, model_name: str, dtype: str = "float16", device: Optional[str] = None,
                 attn_implementation: str = "eager"):
        from transformers import AutoModelForCausalLM, AutoTokenizer
        torch_dtype = _DTYPE_MAP[dtype]
        self.device = torch.device(device) if device else (
            torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu"))
        self.tokenizer = AutoTokenizer.from_pretrained(model_name)
        model = AutoModelForCausalLM.from_pretrained(
            model_name, torch_dtype=torch_dtype, attn_implementation=attn_implementation,
            low_cpu_mem_usage=True).to(self.device).eval()
        self._init_from(model, self.tokenizer)

    @classmethod
    def from_hf(cls, model, tokenizer=None) -> "LayerwiseModel":
        """Wrap an already-loaded HF model (no download)."""
        self = cls.__new__(cls)
        self._init_from(model, tokenizer)
        return self

    def _init_from(self, model, tokenizer):
        self.model = model
        self.tokenizer = tokenizer
        p = next(model.parameters())
        self.device = p.device
        self.dtype = p.dtype
        self._inner = model.model
        self.num_layers = len(self._inner.layers)
        self._pre_rope_k: dict[int, torch.Tensor] = {}
        self._hook_handles: list = []
        self._install_k_proj_hooks()

    def fused_projections(self, layer_idx: int):
        """(W_qkv, W_gate_up) of decoder layer ``layer_idx``: the q/k/v and the
        gate/up projection weights stacked along the output dimension, so one
        GEMM computes each group (at a few hundred to a few thousand rows, or
        one decode row, a single GEMM is faster than its parts).  On first use
        the modules' own weights become row views of the stacked ones -- same
        values, no second copy; a state dict taken afterwards holds views of
        one buffer per group.  An entry is None where the layer's projections
        are not bias-free nn.Linear modules of one input size."""
        fused = getattr(self, "_fused", None)
        if fused is None:
            fused = []
            with torch.inference_mode(False), torch.no_grad():
                for layer in self._inner.layers:
                    attn, mlp = layer.self_attn, getattr(layer, "mlp", None)
                    qkv = [getattr(attn, n, None) for n in ("q_proj", "k_proj", "v_proj")]
                    gu = [getattr(mlp, n, None) for n in ("gate_proj", "up_proj")]
                    fused.append((_stack_linear(qkv) if all(m is not None for m in qkv) else None,
                                  _stack_linear(gu) if all(m is not None for m in gu) else None))
            self._fused = fused
        return fused[layer_idx]

    # -- hooks ----------------------------------------------------------------
    def _install_k_proj_hooks(self) -> None:
        for idx, layer in enumerate(self._inner.layers):
            def hook(_m, _inp, out, _idx=idx):
                self._pre_rope_k[_idx] = out.detach()
            self._hook_handles.append(layer.self_attn.k_proj.register_forward_hook(hook))

    # -- the seven methods ----------------------------------------------------
    def embed_tokens(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self._inner.embed_tokens(input_ids)

    def compute_position_embeddings(self, hidden_states: torch.Tensor, position_ids: torch.Tensor):
        return self._inner.rotary_emb(hidden_states, position_ids)

    def _attn_impl(self) -> str:
        return getattr(self.model.config, "_attn_implementation", None) or "eager"

    def build_causal_mask(self, input_ids: torch.Tensor, position_ids=None, past_key_values=None):
        """Additive causal mask for eager attention; None when the attention
        implementation applies causality itself (sdpa / flash)."""
        S = input_ids.shape[-1]
        past = past_key_values.get_seq_length() if past_key_values is not None else 0
        return self._causal_mask(S, past, self.embed_tokens(input_ids).dtype, input_ids.device)

    def _causal_mask(self, S: int, past: int, dtype, device):
        if self._attn_impl() != "eager":
            return None
        mask = torch.zeros((1, 1, S, past + S), dtype=dtype, device=device)
        future = torch.ones((S, past + S), dtype=torch.bool, device=device).triu(diagonal=past + 1)
        return mask.masked_fill_(future, float("-inf"))

    def prefill_layer(self, layer_idx: int, hidden_states: torch.Tensor, position_ids: torch.Tensor,
                      attention_mask, past_key_values=None, position_embeddings=None,
                      cache_position=None) -> torch.Tensor:
        layer = self._inner.layers[layer_idx]
        if position_embeddings is None:
            position_embeddings = self.compute_position_embeddings(hidden_states, position_ids)
        if cache_position is None:
            past = past_key_values.get_seq_length() if past_key_values is not None else 0
            cache_position = torch.arange(past, past + hidden_states.shape[1], device=hidden_states.device)
        out = layer(hidden_states=hidden_states, attention_mask=attention_mask,
                    position_ids=position_ids, past_key_values=past_key_values,
                    use_cache=past_key_values is not None, cache_position=cache_position,
                    position_embeddings=position_embeddings)
        return out[0] if isinstance(out, tuple) else out

    def final_norm_and_lm_head(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self.model.lm_head(self._inner.norm(hidden_states))

    def forward_layerwise(self, input_ids: torch.Tensor, attention_mask=None, position_ids=None,
                          use_cache: bool = True) -> LayerwiseOutput:
        """Full forward, layer by layer, like the HF model's own forward."""
        self._pre_rope_k = {}
        cache = new_dynamic_cache() if use_cache else None
        h = self.embed_tokens(input_ids)
        S = h.shape[1]
        if position_ids is None:
            past = cache.get_seq_length() if cache is not None else 0
            cache_position = torch.arange(past, past + S, device=h.device)
            position_ids = cache_position.unsqueeze(0)
        else:
            start = int(position_ids.min().item())
            cache_position = torch.arange(start, start + S, device=h.device)
        mask = attention_mask if attention_mask is not None else self._causal_mask(S, 0, h.dtype, h.device)
        pe = self.compute_position_embeddings(h, position_ids)
        for li in range(self.num_layers):
            h = self.prefill_layer(li, h, position_ids, mask, cache, pe, cache_position)
        return LayerwiseOutput(logits=self.final_norm_and_lm_head(h), past_key_values=cache)

    def get_pre_rope_k(self, layer_idx: int) -> torch.Tensor:
        if layer_idx not in self._pre_rope_k:
            raise KeyError(f"No pre-RoPE K for layer {layer_idx}. Run forward_layerwise() first. "
                           f"Available: {sorted(self._pre_rope_k.keys())}")
        return self._pre_rope_k[layer_idx]

    def __del__(self):
        for h in getattr(self, "_hook_handles", []):
            try:
                h.remove()
            except Exception:
                pass
