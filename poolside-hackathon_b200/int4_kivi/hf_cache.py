"""HuggingFace `Cache` backed by the INT4-KIVI store (the reference's
int4_kivi/hf_cache.py:41-267 contract, on libkivi_sm100 kernels).

Per layer: completed 16-token pages are frozen into INT4 with `store_kivi`
semantics (K per-channel, V per-token); the partial page stays bf16.  `update`
returns the full dequantised bf16 K/V `[B, H, S, D]` so the model's own
attention runs unchanged.  The reference takes batch 1 only; here a batch of
B sequences (equal lengths, as `generate` keeps them) is stored as B*H
stacked heads, which every kernel of the library takes as is, so each
sequence's pages and outputs are the ones it would get alone.  Sliding-window layers keep only the trailing
window, exactly as DynamicSlidingWindowLayer does.

B200 differences (values returned are identical):
  * frozen pages live in ONE capacity-backed packed cache per layer and new
    pages are appended in place (`append_kivi`), instead of a list of chunks;
  * the dequantised prefix is kept in a grow-only bf16 buffer and only newly
    frozen pages are dequantised per step, instead of every chunk on every
    step (hf_cache.py:137-154 re-dequantised O(S) bytes per token).

Fused read path (`Int4KiviCache(config, fused_decode=True)` together with
`enable_fused_decode(model)`): single-token steps of full-attention layers do
not materialise bf16 K/V at all.  `update` stores the token and returns an
empty placeholder tagged with its layer; the "int4_kivi" attention function
then runs the fused decode on the packed pages plus the bf16 partial page
(K and V both unquantised, as `update` would have returned them).  Steps of
up to FUSED_MAX_Q tokens (a speculative verify step) take the multi-query
decode, each query at its causal position.  Prefill
and sliding-window layers keep the dequantise + SDPA path, with the
dequantised prefix built per call instead of kept, so the cache holds only
packed pages and at most 15 bf16 tokens per layer.
"""
from __future__ import annotations

import torch
from torch import Tensor

from transformers.cache_utils import Cache, CacheLayerMixin

from .cache import BLOCK, KIVICache, alloc_packed, append_kivi, dequant_kivi, store_kivi
from .mixed import store_kivi_int3v

ATTN_IMPL = "int4_kivi"
# Steps of up to this many new tokens (a decode step, or a speculative verify
# step) take the fused read path; longer ones (prefill) take SDPA.
FUSED_MAX_Q = 8


class _Int4KiviLayer(CacheLayerMixin):
    def __init__(self, k_calib: str = "mse", v_calib: str = "mse", is_sliding: bool = False,
                 sliding_window: int | None = None, fused_decode: bool = False, v_bits: int = 4):
        super().__init__()
        if v_bits not in (3, 4):
            raise ValueError(f"v_bits must be 4 (INT4 KIVI) or 3 (INT4 K / INT3 V), not {v_bits}")
        self.k_calib, self.v_calib, self.v_bits = k_calib, v_calib, v_bits
        self.is_sliding, self.sliding_window = is_sliding, sliding_window
        self.fused = fused_decode and not is_sliding
        self.store: KIVICache | None = None     # frozen pages (S multiple of 16)
        self.hot_k: Tensor | None = None        # [B*H, t < 16, D] bf16 (sequence-major heads)
        self.hot_v: Tensor | None = None
        self.cumulative_length = 0
        self._offset = 0                        # frozen tokens dropped by sliding eviction
        self._deq_k: Tensor | None = None       # [B*H, cap, D] bf16 dequantised frozen prefix
        self._deq_v: Tensor | None = None
        self._deq_len = 0

    # -- transformers Cache layer interface ---------------------------------
    def lazy_initialization(self, key_states: Tensor, value_states: Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        self.is_initialized = True

    def get_max_cache_shape(self) -> int:
        return self.sliding_window if self.is_sliding else -1

    def get_seq_length(self) -> int:
        return self.cumulative_length if self.is_sliding else self._stored_len()

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        if not self.is_sliding:
            return self.get_seq_length() + query_length, 0
        is_full = self.cumulative_length >= self.sliding_window
        kv_offset = max(self.cumulative_length - self.sliding_window + 1, 0)
        kv_length = self.sliding_window - 1 + query_length if is_full else self.cumulative_length + query_length
        return kv_length, kv_offset

    # -- internals -----------------------------------------------------------
    def _hot_len(self) -> int:
        return 0 if self.hot_k is None else self.hot_k.shape[1]

    def _frozen_len(self) -> int:
        return (0 if self.store is None else self.store.S) - self._offset

    def _stored_len(self) -> int:
        return self._frozen_len() + self._hot_len()

    def _freeze_pages(self) -> None:
        n_full = (self._hot_len() // BLOCK) * BLOCK
        if n_full == 0:
            return
        kp, vp = self.hot_k[:, :n_full], self.hot_v[:, :n_full]
        if self.store is None:
            store = store_kivi if self.v_bits == 4 else store_kivi_int3v
            self.store = store(kp.contiguous(), vp.contiguous(), self.k_calib, self.v_calib,
                               capacity=max(4 * n_full, 1024))
        else:
            append_kivi(self.store, kp, vp, self.k_calib, self.v_calib)
        self.hot_k = self.hot_k[:, n_full:].contiguous()
        self.hot_v = self.hot_v[:, n_full:].contiguous()

    def _evict_sliding(self, n_new: int) -> None:
        """Drop whole pages from the front while the stored tokens still cover
        what `get_mask_sizes` promises (window - 1 + the tokens of this call,
        with one page of slack for the next call)."""
        if not self.is_sliding or self.store is None:
            return
        keep = self.sliding_window - 1 + max(BLOCK, n_new)
        while self._frozen_len() >= BLOCK and self._stored_len() - BLOCK >= keep:
            self._offset += BLOCK       # view offset
        if self._offset >= 2048 and self._offset >= self._frozen_len():
            self._compact()

    def _compact(self) -> None:
        """Move the retained pages to the front of a fresh buffer so evicted
        pages do not accumulate over a long sliding-window generation."""
        c, off = self.store, self._offset
        S1 = c.S - off
        kp, ks, vp, vs = alloc_packed(c.H, S1, c.D, c.k_packed.device, c.k_scale.dtype, s_cap=max(4 * S1, 1024),
                                      v_pack=c.v_packed.shape[3])
        NP1 = S1 // BLOCK
        kp[:, :, :NP1].copy_(c.k_packed[:, :, off // BLOCK:])
        ks[:, :, :NP1].copy_(c.k_scale[:, :, off // BLOCK:])
        vp[:, :S1].copy_(c.v_packed[:, off:])
        vs[:, :S1].copy_(c.v_scale[:, off:])
        self.store = type(c)(k_packed=kp[:, :, :NP1], k_scale=ks[:, :, :NP1], k_hot=c.k_hot,
                             v_packed=vp[:, :S1], v_scale=vs[:, :S1], H=c.H, S=S1, D=c.D)
        self._offset = 0
        self._deq_k = self._deq_v = None
        self._deq_len = 0

    def _dequant_frozen(self) -> tuple[Tensor, Tensor]:
        S = 0 if self.store is None else self.store.S
        if self.fused:                      # no persistent bf16 copy in fused mode
            k_all, v_all = dequant_kivi(self.store)
            return k_all[:, self._offset:S], v_all[:, self._offset:S]
        if S > self._deq_len:
            k_all, v_all = dequant_kivi(self.store)   # newly frozen pages only are kept below
            H, _, D = k_all.shape
            if self._deq_k is None or self._deq_k.shape[1] < S:
                cap = max(2 * S, 1024)
                nk = torch.empty((H, cap, D), dtype=torch.bfloat16, device=k_all.device)
                nv = torch.empty_like(nk)
                if self._deq_len:
                    nk[:, :self._deq_len] = self._deq_k[:, :self._deq_len]
                    nv[:, :self._deq_len] = self._deq_v[:, :self._deq_len]
                self._deq_k, self._deq_v = nk, nv
            self._deq_k[:, self._deq_len:S] = k_all[:, self._deq_len:S]
            self._deq_v[:, self._deq_len:S] = v_all[:, self._deq_len:S]
            self._deq_len = S
        return self._deq_k[:, self._offset:S], self._deq_v[:, self._offset:S]

    # -- the contract the model calls ----------------------------------------
    def update(self, key_states: Tensor, value_states: Tensor, *args, **kwargs) -> tuple[Tensor, Tensor]:
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        B, H, n_new, D = key_states.shape
        if self.hot_k is not None and (B, H, D) != (self._B, self._H, self._D):
            raise ValueError(f"batch/heads/head_dim changed from {(self._B, self._H, self._D)} to {(B, H, D)}")
        self._B, self._H, self._D = B, H, D
        k_new = key_states.to(torch.bfloat16).reshape(B * H, n_new, D)
        v_new = value_states.to(torch.bfloat16).reshape(B * H, n_new, D)
        self.cumulative_length += n_new
        if self.hot_k is None:
            self.hot_k, self.hot_v = k_new, v_new
        else:
            self.hot_k = torch.cat([self.hot_k, k_new], dim=1)
            self.hot_v = torch.cat([self.hot_v, v_new], dim=1)
        self._freeze_pages()
        self._evict_sliding(n_new)
        if self.fused and n_new <= FUSED_MAX_Q:
            # the "int4_kivi" attention function reads the packed pages itself
            stub = torch.empty((B, H, 0, D), dtype=torch.bfloat16, device=k_new.device)
            stub._kivi_layer = self
            return stub, stub
        return self._dense_kv(n_new)

    def _dense_kv(self, n_new: int) -> tuple[Tensor, Tensor]:
        """bf16 K/V [B, H, S, D] of everything stored (sliding layers: the
        window the mask of a call with `n_new` tokens expects)."""
        ks, vs = [], []
        if self._frozen_len() > 0:
            fk, fv = self._dequant_frozen()
            ks.append(fk); vs.append(fv)
        if self._hot_len() > 0:
            ks.append(self.hot_k); vs.append(self.hot_v)
        k_full = torch.cat(ks, dim=1) if len(ks) > 1 else ks[0]
        v_full = torch.cat(vs, dim=1) if len(vs) > 1 else vs[0]
        if self.is_sliding and self.cumulative_length >= self.sliding_window:
            want = self.sliding_window - 1 + n_new
            if k_full.shape[1] > want:
                k_full, v_full = k_full[:, -want:], v_full[:, -want:]
        B, H = self._B, self._H
        return k_full.view(B, H, *k_full.shape[1:]), v_full.view(B, H, *v_full.shape[1:])

    def fused_decode(self, query: Tensor, scaling: float | None) -> Tensor:
        """Attention of the step's query tokens over everything stored, each
        query at its causal position (the last q_len stored tokens are the
        step's own): query [B, Hq, q_len, D] -> bf16 [B, Hq, D] for q_len 1,
        else [B, q_len, Hq, D]."""
        from .decode import decode_packed, kivi_decode_attention_multiquery
        Hq, D = query.shape[1], query.shape[3]
        frozen, t = self._frozen_len(), self._hot_len()
        c = self.store
        st = dict(k_packed=c.k_packed if frozen else None, k_scale=c.k_scale if frozen else None,
                  v_packed=c.v_packed if frozen else None, v_scale=c.v_scale if frozen else None,
                  k_hot=self.hot_k if t else torch.empty((self._B * self._H, 0, D), dtype=torch.bfloat16,
                                                         device=query.device),
                  H=self._H, S=frozen + t, D=D, B=self._B, fmt="int4" if self.v_bits == 4 else "int4k_int3v")
        if query.shape[2] > 1:
            return kivi_decode_attention_multiquery(query.transpose(1, 2).to(torch.bfloat16), st, Hq,
                                                    sm_scale=scaling, v_hot=self.hot_v if t else None)
        q = query[:, :, 0].to(torch.bfloat16)
        return decode_packed(q, st, Hq, sm_scale=scaling, v_hot=self.hot_v if t else None)

    # -- memory accounting ----------------------------------------------------
    def nbytes(self) -> int:
        total = 0
        if self.store is not None and self._frozen_len() > 0:
            per_tok = self.store.nbytes / max(self.store.S, 1)
            total += int(per_tok * self._frozen_len())
        if self.hot_k is not None:
            total += self.hot_k.numel() * self.hot_k.element_size() * 2
        return total

    def bf16_nbytes(self) -> int:
        heads = getattr(self, "_B", 0) * getattr(self, "_H", 0)
        return 2 * (self._stored_len() * heads * getattr(self, "_D", 0)) * 2

    def reset(self) -> None:
        self.__init__(self.k_calib, self.v_calib, self.is_sliding, self.sliding_window, self.fused, self.v_bits)

    def reorder_cache(self, beam_idx) -> None:
        if getattr(self, "_B", 1) > 1:
            raise NotImplementedError("beam reordering is not supported by Int4KiviCache")

    def crop(self, max_length: int) -> None:
        raise NotImplementedError("crop is not supported by Int4KiviCache")

    def batch_repeat_interleave(self, repeats: int) -> None:
        raise NotImplementedError("batch expansion is not supported by Int4KiviCache")

    def batch_select_indices(self, indices) -> None:
        raise NotImplementedError("batch selection is not supported by Int4KiviCache")


class Int4KiviCache(Cache):
    """Drop-in ``past_key_values`` for ``model.generate``:

        cache = Int4KiviCache(config=model.config)
        model.generate(..., past_key_values=cache)

    v_bits=3 keeps V in INT3 (the mixed cache of int4_kivi.mixed: 144 bytes
    per token and kv-head instead of 160).
    """

    def __init__(self, config, k_calib: str = "mse", v_calib: str = "mse", fused_decode: bool = False,
                 v_bits: int = 4):
        decoder = config.get_text_config(decoder=True)
        sliding_window = getattr(decoder, "sliding_window", None) or getattr(decoder, "attention_chunk_size", None)
        layer_types = getattr(decoder, "layer_types", None)
        if layer_types is None:
            kind = "sliding_attention" if sliding_window is not None else "full_attention"
            layer_types = [kind] * decoder.num_hidden_layers
        layers = [_Int4KiviLayer(k_calib=k_calib, v_calib=v_calib, is_sliding=(lt == "sliding_attention"),
                                 sliding_window=sliding_window if lt == "sliding_attention" else None,
                                 fused_decode=fused_decode, v_bits=v_bits)
                  for lt in layer_types]
        super().__init__(layers=layers)

    def update(self, key_states: Tensor, value_states: Tensor, layer_idx: int, *args, **kwargs):
        if layer_idx == 0 and key_states.is_cuda:
            # once per forward step: raise a device error flag set by an
            # earlier step's kernels (sync-free, see _native.poll_errors)
            from . import _native
            _native.poll_errors(key_states.device)
        return super().update(key_states, value_states, layer_idx, *args, **kwargs)

    def nbytes(self) -> int:
        return sum(l.nbytes() for l in self.layers)

    def bf16_nbytes(self) -> int:
        return sum(l.bf16_nbytes() for l in self.layers)

    def compression_ratio_vs_bf16(self) -> float:
        return self.bf16_nbytes() / max(self.nbytes(), 1)


def kivi_attention_forward(module, query: Tensor, key: Tensor, value: Tensor, attention_mask, dropout: float = 0.0,
                           scaling: float | None = None, **kwargs):
    """transformers attention function ("int4_kivi"): placeholders from a fused
    Int4KiviCache layer go to the fused decode; anything else (prefill,
    sliding layers, no cache) to the stock SDPA function.  A mask that hides
    any stored position (a left-padded batch) also takes SDPA, over the
    layer's dequantised K/V, since the fused decode attends to every token."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    layer = getattr(key, "_kivi_layer", None)
    q_len = query.shape[2]
    if layer is not None and not _causal_over_all(attention_mask, q_len):
        key, value = layer._dense_kv(q_len)
        layer = None
    if layer is None:
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, **kwargs)
    out = layer.fused_decode(query, scaling)              # [B, Hq, D] or [B, q_len, Hq, D]
    if q_len == 1:
        out = out[:, None]
    return out.to(query.dtype), None                      # [B, q_len, Hq, D]


_mask_memo: list = [None, -1, True]   # [mask tensor of the last check, its version, its result]


def _causal_over_all(mask, q_len: int) -> bool:
    """True when `mask` (None, bool where True attends, or additive float,
    [B, 1, q_len, kv_len]) is the plain causal mask over every stored key:
    query j sees keys 0 .. kv_len - q_len + j and nothing is padded.  That is
    what the fused path computes.  Every layer of one forward step gets the
    same mask tensor, so the answer (which needs a device-to-host read) is
    computed once per step and reused for the other layers."""
    if mask is None:
        return True
    if _mask_memo[0] is mask and _mask_memo[1] == mask._version:
        return _mask_memo[2]
    allowed = mask if mask.dtype == torch.bool else (mask == 0)
    kv, nq = allowed.shape[-1], allowed.shape[-2]
    j = torch.arange(nq, device=allowed.device)[:, None]
    t = torch.arange(kv, device=allowed.device)[None, :]
    ok = nq == q_len and bool((allowed == (t <= kv - nq + j)).all())
    _mask_memo[:] = [mask, mask._version, ok]
    return ok


def enable_fused_decode(model) -> None:
    """Register the "int4_kivi" attention function and switch `model` to it;
    pair with `Int4KiviCache(model.config, fused_decode=True)`.  The name also
    gets SDPA's mask builder: without one, transformers passes no mask at all
    to an unknown attention name, which would drop a batch's padding."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(ATTN_IMPL, kivi_attention_forward)
    AttentionMaskInterface.register(ATTN_IMPL, sdpa_mask)
    model.set_attn_implementation(ATTN_IMPL)
