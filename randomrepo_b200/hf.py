"""HF transformers models (Qwen2 family) decoding and prefilling through the paged KV store.

AgentRL's continuous-batching loop (agentrl/generation/continuous.py:363-504)
keeps one HF ``DynamicCache`` per sequence, stacks the caches of a length
bucket, runs the model forward over one token and splits the caches again,
every step.  Here the paged store is the cache:

* ``register()`` adds the attention implementation ``"paged_b200"`` to HF's
  ``AttentionInterface``.  A model switched to it runs its projections,
  rotary embeddings and MLPs unchanged; each attention layer hands its fresh
  q/k/v to the store, which appends k/v into the pages and attends over them
  (``decode_attention`` for a decode step, ``prefill_attention`` for packed
  prompt chunks).  HF builds no causal mask for an implementation it has no
  mask function for, and no HF cache is passed, so nothing else is stored.
* ``PagedGenerator`` is the rollout loop on top: packed (and chunked) prefill
  of many prompts in one forward, copy-on-write forks of a GRPO group's
  prompt pages, and decode steps over all active sequences at once (one
  allocator step, one forward, no length buckets and no per-sequence cache
  stacking), with greedy or temperature / top-p sampling as in
  agentrl/core/rollout.py:307-329.

With ``cuda_graphs=True`` a decode step's whole forward (all layers, the
attention launches and the LM head) is recorded once per batch size in a CUDA
graph and replayed: the store runs in fixed-step mode (each step's descriptor
goes to one device block whose header the kernels read), so a step costs the
allocator step, one small upload and one graph launch on the host instead of
a Python forward through every layer.  Graphs exist for a fixed ladder of
batch sizes (``GRAPH_BATCHES``); a step of fewer sequences is padded with
placeholder sequences (each holding at most one block, rolled back when it
fills), so a batch that shrinks as sequences finish reuses its graphs.

Only ``last_hidden_state`` rows that need logits go through the LM head, so a
long packed prefill never materialises [tokens, vocab] logits.  By default
the head's logits come out in fp32 (a 16-bit GEMM accumulating and storing in
fp32 on the GPU): a 16-bit head rounds logits to 8 bits of mantissa, which
leaves exact ties in the argmax and coarse log-probabilities for the trainer.
"""

from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass, field

import numpy as np
import torch

from .sampling import SamplingConfig, top_p_filter

ATTN_IMPLEMENTATION = "paged_b200"

_local = threading.local()


@dataclass
class _Phase:
    kind: str                    # "decode" or "prefill"
    store: object
    step: object = None          # DecodeStep (decode) or PrefillStep (prefill, laid out by the first layer)
    sequence_ids: list = field(default_factory=list)
    q_lens: np.ndarray | None = None


@contextlib.contextmanager
def _phase(ph: _Phase):
    prev = getattr(_local, "phase", None)
    _local.phase = ph
    try:
        yield
    finally:
        _local.phase = prev


def _paged_rows(ph: _Phase, layer: int, q, k, v, b: int, t: int, scaling):
    """The store's attention for q [b*t, Hq, D], k/v [b*t, Hkv, D] (contiguous) -> [b*t, Hq, D]."""
    hq = q.shape[1]
    if ph.kind == "decode":
        if t != 1:
            raise ValueError("a decode step feeds one token per sequence")
        return ph.store.decode_attention(ph.step, layer, q, k, v, scale=scaling)
    if b != 1 and (ph.q_lens is None or len(ph.q_lens) != b or any(int(n) != t for n in ph.q_lens)):
        raise ValueError("prefill runs packed (batch 1, the chunks of all sequences along the token axis) or as a "
                         "batch of equal chunks, one per sequence")
    if ph.step is None and hasattr(ph.store, "prefill_step"):
        ph.step = ph.store.prefill_step(ph.sequence_ids, ph.q_lens, hq)
    return ph.store.prefill_attention(ph.sequence_ids, q, k, v, q_lens=ph.q_lens, layer=layer, scale=scaling,
                                      step=ph.step)


def paged_attention_forward(module, query, key, value, attention_mask=None, scaling=None, dropout=0.0, **kwargs):
    """HF attention-interface entry: q [B, Hq, T, D], k/v [B, Hkv, T, D] -> ([B, T, Hq, D], None)."""
    ph = getattr(_local, "phase", None)
    if ph is None:
        # A forward of an HF model over a PagedCache(kernels=True): set up by the cache at layer 0,
        # valid for that forward's layers only.
        ph = getattr(_local, "cache_phase", None)
        if ph is not None:
            _local.cache_layers_left -= 1
            if _local.cache_layers_left <= 0:
                _local.cache_phase = None
    if ph is None:
        raise RuntimeError("paged_b200 attention ran outside a PagedGenerator forward or a PagedCache(kernels=True)")
    b, hq, t, d = query.shape
    hkv = key.shape[1]
    out = _paged_rows(ph, int(module.layer_idx), query.transpose(1, 2).reshape(b * t, hq, d).contiguous(),
                      key.transpose(1, 2).reshape(b * t, hkv, d).contiguous(),
                      value.transpose(1, 2).reshape(b * t, hkv, d).contiguous(), b, t, scaling)
    return out.view(b, t, hq, d), None


# -- fused layers ---------------------------------------------------------------
# Inside a PagedGenerator forward, the decoder layers of a Qwen2-family model
# on the GPU (bf16 / f16, SiLU MLP) run their RMSNorms (with the residual add
# folded into the second), rotary embedding and SiLU product as single
# launches of the library (pkv_rms_norm, pkv_rope, pkv_silu_mul) instead of
# HF's eager op chains; q / k / v come from one GEMM over the three
# projections' weights and gate / up from one over the MLP's two (the
# parameters become views into those packed weights: no extra memory, HF's
# modules see the same values), the MLP's residual add rides in the down
# projection's GEMM (addmm), and the rotated q / k reach the store without
# the HF layout transposes.  Outside such a forward every module runs its own
# HF code unchanged.

def _dtype_code(t: torch.Tensor) -> int:
    from ._lib import PKV_BF16, PKV_F16

    return PKV_BF16 if t.dtype == torch.bfloat16 else PKV_F16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def fused_rms_norm(x: torch.Tensor, norm, residual: torch.Tensor | None = None):
    """``norm(x)`` (a Qwen2RMSNorm) in one launch; with ``residual``, of ``residual + x``, which is returned too."""
    from ._lib import lib, raise_for_status

    x = x.contiguous()
    hidden = x.shape[-1]
    out = torch.empty_like(x)
    total = None
    if residual is not None:
        residual = residual.contiguous()
        total = torch.empty_like(x)
    raise_for_status(lib.pkv_rms_norm(x.data_ptr(), residual.data_ptr() if residual is not None else None,
                                      total.data_ptr() if total is not None else None, norm.weight.data_ptr(),
                                      out.data_ptr(), x.numel() // hidden, hidden, float(norm.variance_epsilon),
                                      _dtype_code(x), _stream()))
    return out if residual is None else (out, total)


def fused_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, head_dim: int):
    """apply_rotary_pos_emb on the projections' outputs q [..., Hq*D], k [..., Hkv*D] -> [rows, H, D] each."""
    from ._lib import lib, raise_for_status

    rows = q.numel() // q.shape[-1]
    hq, hkv = q.shape[-1] // head_dim, k.shape[-1] // head_dim
    q = q.contiguous()
    k = k.contiguous()
    cos = cos.contiguous()
    sin = sin.contiguous()
    qo = torch.empty((rows, hq, head_dim), dtype=q.dtype, device=q.device)
    ko = torch.empty((rows, hkv, head_dim), dtype=k.dtype, device=k.device)
    raise_for_status(lib.pkv_rope(q.data_ptr(), k.data_ptr(), None, cos.data_ptr(), sin.data_ptr(), qo.data_ptr(),
                                  ko.data_ptr(), None, rows, hq * head_dim, hkv * head_dim, 0, hq, hkv, head_dim,
                                  _dtype_code(q), _stream()))
    return qo, ko


def fused_rope_qkv(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, hq: int, hkv: int, head_dim: int):
    """One packed projection row per token, [..., (Hq + 2 Hkv) * D] = q | k | v -> rotated q [rows, Hq, D],
    rotated k and v [rows, Hkv, D], contiguous."""
    from ._lib import lib, raise_for_status

    ld = qkv.shape[-1]
    rows = qkv.numel() // ld
    qkv = qkv.contiguous()
    cos = cos.contiguous()
    sin = sin.contiguous()
    qo = torch.empty((rows, hq, head_dim), dtype=qkv.dtype, device=qkv.device)
    ko = torch.empty((rows, hkv, head_dim), dtype=qkv.dtype, device=qkv.device)
    vo = torch.empty((rows, hkv, head_dim), dtype=qkv.dtype, device=qkv.device)
    esz = qkv.element_size()
    base = qkv.data_ptr()
    raise_for_status(lib.pkv_rope(base, base + hq * head_dim * esz, base + (hq + hkv) * head_dim * esz,
                                  cos.data_ptr(), sin.data_ptr(), qo.data_ptr(), ko.data_ptr(), vo.data_ptr(), rows,
                                  ld, ld, ld, hq, hkv, head_dim, _dtype_code(qkv), _stream()))
    return qo, ko, vo


def fused_silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SiLU(gate) * up in one launch (both [..., cols], contiguous)."""
    from ._lib import lib, raise_for_status

    gate = gate.contiguous()
    up = up.contiguous()
    cols = gate.shape[-1]
    out = torch.empty_like(gate)
    raise_for_status(lib.pkv_silu_mul(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel() // cols, cols,
                                      cols, _dtype_code(gate), _stream()))
    return out


def fused_silu_mul_packed(gate_up: torch.Tensor) -> torch.Tensor:
    """SiLU(gate) * up from one packed row [..., 2 * I] = gate | up -> [rows, I]."""
    from ._lib import lib, raise_for_status

    gate_up = gate_up.contiguous()
    ld = gate_up.shape[-1]
    cols = ld // 2
    rows = gate_up.numel() // ld
    out = torch.empty((rows, cols), dtype=gate_up.dtype, device=gate_up.device)
    base = gate_up.data_ptr()
    raise_for_status(lib.pkv_silu_mul(base, base + cols * gate_up.element_size(), out.data_ptr(), rows, cols, ld,
                                      _dtype_code(gate_up), _stream()))
    return out


def _fused_norm_forward(self, hidden_states):
    if getattr(_local, "phase", None) is None:
        return type(self).forward(self, hidden_states)
    return fused_rms_norm(hidden_states, self)


def _fused_mlp_forward(self, x):
    if getattr(_local, "phase", None) is None:
        return type(self).forward(self, x)
    act = fused_silu_mul_packed(torch.nn.functional.linear(x, _gate_up(self)))
    return self.down_proj(act).view(*x.shape[:-1], -1)


def _is_view_at(t: torch.Tensor | None, packed: torch.Tensor | None, offset: int) -> bool:
    """Whether ``t`` still lies at element ``offset`` of ``packed`` (same dtype and device)."""
    if t is None or packed is None:
        return t is None and packed is None
    return (t.dtype == packed.dtype and t.device == packed.device
            and t.data_ptr() == packed.data_ptr() + offset * packed.element_size())


def _gate_up(mlp) -> torch.Tensor:
    """The packed gate | up weight, packed again if either parameter was re-allocated (moved, cast,
    or replaced on its own, e.g. by a weight sync that sets ``.data`` of one projection)."""
    gu = mlp._pkv_gate_up
    g, u = mlp.gate_proj.weight, mlp.up_proj.weight
    if not (_is_view_at(g, gu, 0) and _is_view_at(u, gu, g.numel()) and g.numel() + u.numel() == gu.numel()):
        with torch.no_grad():
            _pack_gate_up(mlp)
    return mlp._pkv_gate_up


def _qkv_packed(attn) -> bool:
    """Whether every q / k / v weight and bias is still the view of the packed tensors it was made."""
    w, b, _, _ = attn._pkv_qkv
    o = 0
    for p in (attn.q_proj, attn.k_proj, attn.v_proj):
        pw, pb = p.weight, getattr(p, "bias", None)
        if not _is_view_at(pw, w, o * pw.shape[1]):
            return False
        if (pb is None) != (b is None) or (pb is not None and not _is_view_at(pb, b, o)):
            return False
        o += pw.shape[0]
    return o * w.shape[1] == w.numel()


def _fused_mlp_residual(mlp, x, residual):
    """residual + mlp(x), the add done by the down projection's GEMM (addmm, beta = 1)."""
    act = fused_silu_mul_packed(torch.nn.functional.linear(x, _gate_up(mlp)))
    res = residual.reshape(-1, residual.shape[-1])
    return torch.addmm(res, act, mlp.down_proj.weight.t()).view(residual.shape)


def _fused_attention_forward(self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None,
                             **kwargs):
    ph = getattr(_local, "phase", None)
    if ph is None:
        return type(self).forward(self, hidden_states, position_embeddings, attention_mask,
                                  past_key_values=past_key_values, **kwargs)
    input_shape = hidden_states.shape[:-1]
    b, t = int(input_shape[0]), int(input_shape[1])
    d = int(self.head_dim)
    cos, sin = position_embeddings
    if not _qkv_packed(self):
        # A parameter was re-allocated (moved, cast, or replaced on its own): pack them again.
        with torch.no_grad():
            _pack_qkv(self)
    w, bias, hq, hkv = self._pkv_qkv
    qkv = torch.nn.functional.linear(hidden_states, w, bias)
    q, k, v = fused_rope_qkv(qkv, cos, sin, hq, hkv, d)
    out = _paged_rows(ph, int(self.layer_idx), q, k, v, b, t, self.scaling)
    return self.o_proj(out.reshape(*input_shape, -1)), None


def _fused_layer_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                         use_cache=False, position_embeddings=None, **kwargs):
    if getattr(_local, "phase", None) is None:
        return type(self).forward(self, hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                                  past_key_values=past_key_values, use_cache=use_cache,
                                  position_embeddings=position_embeddings, **kwargs)
    h = fused_rms_norm(hidden_states, self.input_layernorm)
    a, _ = self.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                          past_key_values=past_key_values, use_cache=use_cache,
                          position_embeddings=position_embeddings, **kwargs)
    h2, hidden = fused_rms_norm(a, self.post_attention_layernorm, residual=hidden_states)
    if getattr(self.mlp.down_proj, "bias", None) is None:
        return _fused_mlp_residual(self.mlp, h2, hidden)
    return hidden + self.mlp(h2)


def _pack_qkv(attn) -> None:
    """q / k / v weights (and biases) concatenated; the projections' parameters become views into them."""
    projs = (attn.q_proj, attn.k_proj, attn.v_proj)
    d = int(attn.head_dim)
    w = torch.cat([p.weight for p in projs], 0)
    has_bias = all(getattr(p, "bias", None) is not None for p in projs)
    b = torch.cat([p.bias for p in projs], 0) if has_bias else None
    o = 0
    for p in projs:
        n = p.weight.shape[0]
        p.weight.data = w[o:o + n]
        if has_bias:
            p.bias.data = b[o:o + n]
        o += n
    attn._pkv_qkv = (w, b, attn.q_proj.weight.shape[0] // d, attn.k_proj.weight.shape[0] // d)


def _pack_gate_up(mlp) -> None:
    """gate / up weights concatenated; the projections' parameters become views into them."""
    gu = torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0)
    n = mlp.gate_proj.weight.shape[0]
    mlp.gate_proj.weight.data = gu[:n]
    mlp.up_proj.weight.data = gu[n:]
    mlp._pkv_gate_up = gu


def _pack_weights(layer) -> None:
    """q / k / v (and their biases) and gate / up weights concatenated once; the modules' parameters
    become views into the packed tensors (the same values, no extra memory)."""
    if not hasattr(layer.self_attn, "_pkv_qkv"):
        _pack_qkv(layer.self_attn)
    if not hasattr(layer.mlp, "_pkv_gate_up"):
        _pack_gate_up(layer.mlp)


def install_fused_layers(model) -> bool:
    """Give the decoder layers of a Qwen2-family model on the GPU (bf16 / f16) the fused forwards above
    (per instance; the classes are untouched).  Returns whether they were installed."""
    import types

    base = model.get_decoder() if hasattr(model, "get_decoder") else getattr(model, "model", None)
    layers = getattr(base, "layers", None)
    p = next(model.parameters())
    cfg = model.config
    if (layers is None or not p.is_cuda or p.dtype not in (torch.bfloat16, torch.float16)
            or getattr(cfg, "hidden_act", None) != "silu"):
        return False
    for layer in layers:
        attn, mlp = getattr(layer, "self_attn", None), getattr(layer, "mlp", None)
        parts = (getattr(layer, "input_layernorm", None), getattr(layer, "post_attention_layernorm", None))
        if (attn is None or mlp is None or None in parts or not all(hasattr(n, "variance_epsilon") for n in parts)
                or not all(hasattr(attn, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj", "head_dim"))
                or not all(hasattr(mlp, a) for a in ("gate_proj", "up_proj", "down_proj"))
                or getattr(mlp.gate_proj, "bias", None) is not None or getattr(mlp.up_proj, "bias", None) is not None):
            return False
        # q / k / v biases are packed only all together: a model with some of them keeps HF's forwards.
        if len({getattr(p, "bias", None) is None for p in (attn.q_proj, attn.k_proj, attn.v_proj)}) != 1:
            return False
    with torch.no_grad():
        for layer in layers:
            _pack_weights(layer)
    for layer in layers:
        layer.forward = types.MethodType(_fused_layer_forward, layer)
        layer.self_attn.forward = types.MethodType(_fused_attention_forward, layer.self_attn)
        layer.mlp.forward = types.MethodType(_fused_mlp_forward, layer.mlp)
    norm = getattr(base, "norm", None)
    if norm is not None and hasattr(norm, "variance_epsilon"):
        norm.forward = types.MethodType(_fused_norm_forward, norm)
    return True


def register() -> None:
    """Make ``"paged_b200"`` a valid ``config._attn_implementation`` (idempotent)."""
    from transformers import AttentionInterface

    AttentionInterface.register(ATTN_IMPLEMENTATION, paged_attention_forward)


def use_paged_attention(model) -> None:
    """Switch a loaded HF model to the paged attention implementation."""
    register()
    model.config._attn_implementation = ATTN_IMPLEMENTATION
    for sub in model.modules():
        cfg = getattr(sub, "config", None)
        if cfg is not None and cfg is not model.config:
            cfg._attn_implementation = ATTN_IMPLEMENTATION


def kv_geometry(config) -> tuple[int, int, int]:
    """(layers, KV heads, head dim) of a model config, by the rule of
    agentrl/generation/scheduler.py:16-29: KV heads fall back to the attention
    heads, head_dim to hidden_size / attention heads."""
    layers = int(config.num_hidden_layers)
    heads = int(getattr(config, "num_key_value_heads", None) or config.num_attention_heads)
    head_dim = getattr(config, "head_dim", None)
    if head_dim is None:
        head_dim = int(config.hidden_size) // int(config.num_attention_heads)
    return layers, heads, int(head_dim)


def make_store(model, total_blocks: int, block_size: int = 16, device=None):
    """A PagedKVCacheStore shaped for ``model`` (layers, KV heads, head dim, dtype)."""
    from .paged_kv import PagedKVAllocator, PagedKVCacheStore

    layers, heads, head_dim = kv_geometry(model.config)
    dtype = next(model.parameters()).dtype
    dev = device if device is not None else next(model.parameters()).device
    return PagedKVCacheStore(PagedKVAllocator(total_blocks, block_size), num_layers=layers, num_kv_heads=heads,
                             head_dim=head_dim, dtype=dtype, device=dev)


_top_p = top_p_filter

# Batch sizes decode-step graphs are recorded for (multiples of 64 above).
GRAPH_BATCHES = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)


def graph_batch(n: int) -> int:
    """The recorded batch size a decode step of ``n`` sequences is padded to."""
    for b in GRAPH_BATCHES:
        if n <= b:
            return b
    return -(-n // 64) * 64


class PagedGenerator:
    """Rollout loop of a causal LM over the paged store (continuous.py:363-504 without the per-sequence caches).

    Token selection and log-probabilities go through ``sampler`` (by default
    the library's ``DeviceSampler`` kernels, created on first use).  With
    ``fused_layers`` (the default) a Qwen2-family model on the GPU gets the
    fused decoder-layer forwards (``install_fused_layers``): per model
    instance, so a model fused once stays fused for other generators, and
    active only inside these generators' forwards.
    """

    def __init__(self, model, store, *, prefill_chunk_size: int = 512, eos_token_id: int | None = None,
                 fp32_logits: bool = True, cuda_graphs: bool = False, sampler=None, fused_layers: bool = True) -> None:
        use_paged_attention(model)
        # Fused norm / rotary / SiLU launches inside this generator's forwards (Qwen2-family models on the GPU).
        self.fused_layers = bool(fused_layers) and install_fused_layers(model)
        from .device import PinnedStaging

        self._h2d = PinnedStaging()
        self.model = model
        self.store = store
        self.prefill_chunk_size = int(prefill_chunk_size)
        self.eos_token_id = eos_token_id
        self.device = next(model.parameters()).device
        self._base = model.get_decoder() if hasattr(model, "get_decoder") else model.model
        self._head = model.get_output_embeddings()
        self.cuda_graphs = bool(cuda_graphs)
        self._graphs: dict[int, tuple] = {}  # batch -> (graph, static tokens, static positions, static logits)
        self._graph_tables = 0
        self._graph_fixed = 0
        self._pads: list[int] = []           # placeholder sequences that pad graphed steps
        self._pad_len: dict[int, int] = {}
        # (padded batch, chunk length) -> (graph, static ids, static positions, static logits, upload buffers)
        self._ext_graphs: dict[tuple[int, int], tuple] = {}
        self.fp32_logits = bool(fp32_logits)
        self._sampler = sampler
        self._growth_used = 0  # blocks the last admission set aside for its sequences' next tokens
        # Device times of the last generate on a CUDA device: prefill_ms (prompts
        # + forks), decode_ms (the decode loop), token counts.
        self.last_timings: dict = {}

    @property
    def sampler(self):
        if self._sampler is None:
            from .sampling import DeviceSampler

            self._sampler = DeviceSampler(self.device)
        return self._sampler

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """LM head on final hidden states [n, hidden] -> float32 logits [n, vocab]."""
        with torch.inference_mode():
            if not self.fp32_logits:
                return self._head(hidden).float()
            w = self._head.weight
            bias = getattr(self._head, "bias", None)
            if hidden.is_cuda and hidden.dtype == w.dtype and w.dtype in (torch.bfloat16, torch.float16):
                out = torch.mm(hidden, w.t(), out_dtype=torch.float32)
            else:
                out = torch.nn.functional.linear(hidden.float(), w.float())
            return out if bias is None else out + bias.float()

    # -- forwards -------------------------------------------------------------
    def _forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor, ph: _Phase) -> torch.Tensor:
        with _phase(ph), torch.inference_mode():
            out = self._base(input_ids=input_ids, position_ids=position_ids, use_cache=False)
        return out.last_hidden_state

    def _token_count(self, sid: int) -> int:
        return int(self.store.token_count(sid))

    def _token_counts(self, ids) -> list[int]:
        bulk = getattr(self.store, "token_counts", None)
        if bulk is not None:
            return [int(c) for c in bulk(ids)]
        return [self._token_count(s) for s in ids]

    def _append_many(self, ids, counts) -> None:
        bulk = getattr(self.store, "append_many", None)
        if bulk is not None:
            bulk(ids, counts)
        else:
            for sid, n in zip(ids, counts):
                self.store.append_tokens(sid, n)

    def extend_hidden(self, sequence_ids, chunks) -> tuple[torch.Tensor, np.ndarray]:
        """Append one chunk of tokens to each (existing) sequence and run one packed forward
        over all chunks: returns (final hidden states [sum of chunk lengths, hidden], chunk
        lengths).  Each chunk attends to its sequence's cached tokens and causally to itself."""
        ids = [int(s) for s in sequence_ids]
        toks = [torch.as_tensor(c, dtype=torch.long).reshape(-1) for c in chunks]
        if len(ids) != len(toks):
            raise ValueError("one chunk per sequence id")
        q_lens = np.array([t.numel() for t in toks], dtype=np.int64)
        past = self._token_counts(ids)
        self._append_many(ids, [t.numel() for t in toks])
        input_ids = self._h2d.to_device(torch.cat(toks), self.device).unsqueeze(0)
        pos = self._h2d.to_device(torch.cat([torch.arange(p0, p0 + t.numel()) for p0, t in zip(past, toks)]),
                                  self.device)
        h = self._forward(input_ids, pos.unsqueeze(0), _Phase("prefill", self.store, sequence_ids=ids, q_lens=q_lens))
        return h[0], q_lens

    def extend(self, sequence_ids, chunks, *, all_logits: bool = False) -> torch.Tensor:
        """``extend_hidden`` then the LM head: float32 logits of each chunk's last token
        [n, vocab], or of every token [sum of chunk lengths, vocab] with ``all_logits``."""
        h, q_lens = self.extend_hidden(sequence_ids, chunks)
        if all_logits:
            return self.logits(h)
        ends = torch.from_numpy(np.cumsum(q_lens) - 1).to(h.device)
        return self.logits(h.index_select(0, ends))

    def verify_logits(self, sequence_ids, chunks) -> torch.Tensor:
        """Logits of every token of equal-length chunks appended to existing sequences,
        [n * L, vocab] (the speculative verify forward).  With ``cuda_graphs`` the forward is
        replayed from a CUDA graph recorded per (padded batch, L): the step's slots and work
        items go to fixed device buffers, placeholders pad the batch to a recorded size."""
        from . import device as _device
        from ._lib import lib as _lib

        lens = {len(c) for c in chunks}
        cfg = self.model.config
        hq, hkv = int(cfg.num_attention_heads), int(getattr(cfg, "num_key_value_heads", None) or
                                                     cfg.num_attention_heads)
        # The recorded launch needs a fixed shape: every chunk fits one work
        # item per KV head and the plan does not cut keys across CTAs.
        fixed_shape = (len(lens) == 1 and _device.PREFILL_SPLIT_WAVES == 0 and
                       next(iter(lens)) <= _lib.pkv_prefill_positions_per_item(hq, hkv))
        if not self.cuda_graphs or not fixed_shape:
            return self.extend(sequence_ids, chunks, all_logits=True)
        return self._extend_graph([int(s) for s in sequence_ids], chunks, lens.pop())

    def _extend_graph(self, ids, chunks, L: int) -> torch.Tensor:
        store = self.store
        n = len(ids)
        nb = graph_batch(n)
        pads = self._placeholders(nb - n) if nb > n else []
        # _placeholders counted one decode token per placeholder: these take L instead.
        for p in pads:
            self._pad_len[p] -= 1
        past = self._token_counts(ids) + [self._pad_len[p] for p in pads]
        all_ids = ids + pads
        self._append_many(all_ids, [L] * len(all_ids))
        toks = torch.tensor([t for c in chunks for t in c] + [0] * (L * len(pads)), dtype=torch.long)
        pos = torch.tensor([p0 + j for p0 in past for j in range(L)], dtype=torch.long)
        q_lens = np.full(nb, L, dtype=np.int64)
        hq = int(self.model.config.num_attention_heads)
        pool = store.pool
        key = (nb, L)
        entry = self._ext_graphs.get(key)
        try:
            bufs = entry[4] if entry is not None else None
            step = store.prefill_step(all_ids, q_lens, hq, buffers=bufs)
            if pool.tables.data_ptr() != self._graph_tables:
                # The step grew (moved) the device tables: every graph holds the old address.
                self._graphs.clear()
                self._ext_graphs.clear()
                self._graph_tables = pool.tables.data_ptr()
                entry = None
            if entry is None:
                if bufs is None:
                    bufs = {"slots": step.slots.clone(), "records": step.records.clone(),
                            "n_items": step.plan.n_items}
                    step = store.prefill_step(all_ids, q_lens, hq, buffers=bufs)
                tok_s = self._h2d.to_device(toks, self.device).unsqueeze(0)
                pos_s = self._h2d.to_device(pos, self.device).unsqueeze(0)
                ph = _Phase("prefill", store, step=step, sequence_ids=all_ids, q_lens=q_lens)
                cur = torch.cuda.current_stream(self.device)
                side = torch.cuda.Stream(device=self.device)
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    out = self.logits(self._forward(tok_s, pos_s, ph)[0])
                cur.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    logits_s = self.logits(self._forward(tok_s, pos_s, ph)[0])
                self._ext_graphs[key] = (graph, tok_s, pos_s, logits_s, bufs)
            else:
                graph, tok_s, pos_s, logits_s, _ = entry
                tok_s.copy_(self._h2d.to_device(toks, self.device).unsqueeze(0))
                pos_s.copy_(self._h2d.to_device(pos, self.device).unsqueeze(0))
                graph.replay()
                out = logits_s.clone()
        finally:
            if pads:
                store.truncate(pads, [0] * len(pads))
                for p in pads:
                    self._pad_len[p] = 0
        return out[:n * L]

    def prefill(self, sequence_ids, prompts) -> torch.Tensor:
        """Reserve each prompt, write its K/V, return next-token logits [n, vocab] (float32).

        All prompts go through one packed forward per round of chunks of at
        most ``prefill_chunk_size`` tokens (continuous.py:944-976 prefills one
        prompt at a time; prefill.py:65-111 chunks a long one).
        """
        ids = [int(s) for s in sequence_ids]
        toks = [torch.as_tensor(p, dtype=torch.long).reshape(-1) for p in prompts]
        if len(ids) != len(toks):
            raise ValueError("one prompt per sequence id")
        if any(t.numel() == 0 for t in toks):
            raise ValueError("prompts must be non-empty")
        for sid in ids:
            self.store.reserve(sid, 0)
        last_hidden = [None] * len(ids)
        cs = self.prefill_chunk_size
        rounds = max((t.numel() + cs - 1) // cs for t in toks)
        for c in range(rounds):
            members = [i for i, t in enumerate(toks) if t.numel() > c * cs]
            h, q_lens = self.extend_hidden([ids[i] for i in members], [toks[i][c * cs:(c + 1) * cs] for i in members])
            ends = np.cumsum(q_lens) - 1
            for j, i in enumerate(members):
                if (c + 1) * cs >= toks[i].numel():
                    last_hidden[i] = h[int(ends[j])]
        return self.logits(torch.stack(last_hidden))

    def decode_step(self, sequence_ids, tokens: torch.Tensor, *, eager: bool = False) -> torch.Tensor:
        """Feed one token per sequence; returns next-token logits [n, vocab] (float32).  ``eager`` runs
        the step without its CUDA graph (whose placeholder padding could take blocks a full pool lacks)."""
        if self.cuda_graphs and not eager:
            return self._decode_step_graph(sequence_ids, tokens)
        step = self.store.decode_step(sequence_ids)
        pos = self._h2d.to_device(torch.from_numpy(step.host_lens.astype(np.int64) - 1), self.device)
        h = self._forward(self._h2d.to_device(tokens.reshape(-1, 1), self.device) if not tokens.is_cuda
                          else tokens.reshape(-1, 1), pos.reshape(-1, 1),
                          _Phase("decode", self.store, step=step))
        return self.logits(h[:, -1])

    _pad_ids = 1 << 61   # sequence ids of placeholder sequences

    def _placeholders(self, count: int) -> list[int]:
        """``count`` placeholder sequences for padding a graphed step, each with room for one token."""
        while len(self._pads) < count:
            sid = PagedGenerator._pad_ids
            PagedGenerator._pad_ids += 1
            self.store.reserve(sid, 0)
            self._pads.append(sid)
            self._pad_len[sid] = 0
        pads = self._pads[:count]
        bs = self.store.allocator.block_size_tokens
        full = [p for p in pads if self._pad_len[p] >= bs]
        if full:
            self.store.truncate(full, [0] * len(full))
            for p in full:
                self._pad_len[p] = 0
        for p in pads:
            self._pad_len[p] += 1
        return pads

    def release_placeholders(self) -> None:
        """Return the placeholder sequences' rows and blocks to the store."""
        for sid in self._pads:
            if self.store.has_sequence(sid):
                self.store.release(sid)
        self._pads, self._pad_len = [], {}

    def _decode_step_graph(self, sequence_ids, tokens: torch.Tensor) -> torch.Tensor:
        pool = self.store.pool
        n = len(sequence_ids)
        nb = graph_batch(n)
        pads = self._placeholders(nb - n) if nb > n else []
        if pool.fixed_batch < nb:
            pool.fix_steps(max(nb, 2 * pool.fixed_batch))
        step = self.store.decode_step(list(sequence_ids) + pads)
        if pool.tables.data_ptr() != self._graph_tables:
            # Graphs hold the tables' address: a grown (moved) table voids them.
            self._graphs.clear()
            self._ext_graphs.clear()
            self._graph_tables = pool.tables.data_ptr()
        if pool.fixed_serial != self._graph_fixed:
            # Decode graphs hold the fixed step block, which a new capacity replaces.
            self._graphs.clear()
            self._graph_fixed = pool.fixed_serial
        pos = self._h2d.to_device(torch.from_numpy(step.host_lens.astype(np.int64) - 1), self.device)
        tok = tokens.reshape(-1)
        if tok.device != self.device:
            tok = self._h2d.to_device(tok, self.device)
        if pads:
            tok = torch.cat([tok, tok.new_zeros(len(pads))])
        tok = tok.reshape(-1, 1)
        entry = self._graphs.get(nb)
        if entry is None:
            return self._capture(nb, step, tok, pos.reshape(-1, 1))[:n]
        graph, tok_s, pos_s, logits_s = entry
        tok_s.copy_(tok)
        pos_s.copy_(pos.reshape(-1, 1))
        graph.replay()
        return logits_s[:n].clone()

    def _capture(self, n: int, step, tok: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Run this step eagerly (on a side stream, as capture requires a warm-up), then record it."""
        tok_s, pos_s = tok.clone(), pos.clone()
        ph = _Phase("decode", self.store, step=step)
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            logits = self.logits(self._forward(tok_s, pos_s, ph)[:, -1])
        cur.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits_s = self.logits(self._forward(tok_s, pos_s, ph)[:, -1])
        self._graphs[n] = (graph, tok_s, pos_s, logits_s)
        return logits

    def reserve_tables(self, max_tokens: int) -> None:
        """Grow the device tables now for sequences of up to ``max_tokens`` (graph mode keeps their address)."""
        pool = self.store.pool
        stats = self.store.allocator._stats()
        bs = self.store.allocator.block_size_tokens
        pool.grow(int(stats.row_capacity) + 1, -(-int(max_tokens) // bs) + 1)

    # -- old-policy log-probabilities ---------------------------------------------
    _score_ids = 1 << 62   # sequence ids of the scoring pass's temporary sequences

    def score(self, input_ids, attention_mask=None, completion_mask=None, *, group_size: int = 1,
              max_logit_rows: int = 2048) -> torch.Tensor:
        """Per-token log-probabilities of packed sequences (rollout.py:456-472).

        ``input_ids`` / ``attention_mask`` / ``completion_mask`` are [B, L]
        (right padding: each mask row is ones then zeros).  Returns float32
        [B, L] on the model's device: ``out[b, p] = log_softmax(logits[b, p-1])[input_ids[b, p]]``
        where ``completion_mask[b, p]`` is set (p >= 1), else 0 -- the
        reference's aligned ``old_policy_logprobs``.

        The reference runs one full forward over the padded [B, L] batch and a
        log_softmax over [B, L-1, vocab].  Here each group of ``group_size``
        consecutive rows prefills its common prefix once (the members fork
        its pages), the rest of every row goes through packed chunked
        prefill, and logits exist only for rows that are scored, at most
        ``max_logit_rows`` at a time, reduced to one number each by the fused
        log-softmax + gather kernel.
        """
        ids = torch.as_tensor(input_ids).to("cpu", torch.int64)
        if ids.dim() != 2:
            raise ValueError("input_ids must be [B, L]")
        b_rows, width = ids.shape
        am = (torch.ones_like(ids) if attention_mask is None else torch.as_tensor(attention_mask).to("cpu")).bool()
        cm = (torch.ones_like(ids) if completion_mask is None else torch.as_tensor(completion_mask).to("cpu")).bool()
        if am.shape != ids.shape or cm.shape != ids.shape:
            raise ValueError("masks must match input_ids")
        if group_size < 1 or b_rows % group_size:
            raise ValueError("the batch must hold whole groups")
        lens = am.sum(dim=1)
        if not torch.equal(am, torch.arange(width).unsqueeze(0) < lens.unsqueeze(1)):
            raise ValueError("attention_mask must be right padding (ones, then zeros)")
        out = torch.zeros((b_rows, width), dtype=torch.float32, device=self.device)
        rows = [ids[b, :int(lens[b])].tolist() for b in range(b_rows)]
        # Positions p - 1 whose logits are needed (p scored).
        need = [[p - 1 for p in range(1, int(lens[b])) if cm[b, p]] for b in range(b_rows)]
        base = PagedGenerator._score_ids
        PagedGenerator._score_ids += b_rows
        seq = [base + b for b in range(b_rows)]
        try:
            heads = list(range(0, b_rows, group_size))
            shared = {}
            for g0 in heads:
                members = range(g0, g0 + group_size)
                n = min(len(rows[b]) for b in members)
                for b in members:
                    n = next((i for i in range(n) if rows[b][i] != rows[g0][i]), n)
                    if need[b]:
                        n = min(n, need[b][0])
                shared[g0] = n
                self.store.reserve(seq[g0], 0)
            # Every group's common prefix once, all groups packed per round.
            cs = self.prefill_chunk_size
            for c in range(0, max(shared.values()), cs):
                members = [g0 for g0 in heads if shared[g0] > c]
                self.extend_hidden([seq[g0] for g0 in members],
                                   [rows[g0][c:min(c + cs, shared[g0])] for g0 in members])
            for g0 in heads:
                for b in range(g0 + 1, g0 + group_size):
                    self.store.fork(seq[g0], seq[b])
            # Every row's remainder, packed, in rounds of at most prefill_chunk_size tokens per row.
            self._score_rest(seq, rows, need, out, ids, max_logit_rows)
        finally:
            for sid in seq:
                if self.store.has_sequence(sid):
                    self.store.release(sid)
        return out

    def _score_rest(self, seq, rows, need, out, ids, max_logit_rows: int) -> None:
        cs = self.prefill_chunk_size
        pos = self._token_counts(seq)
        need_sets = [set(n) for n in need]
        while True:
            members = [b for b in range(len(seq)) if pos[b] < len(rows[b])]
            if not members:
                return
            chunks = [rows[b][pos[b]:pos[b] + cs] for b in members]
            h, q_lens = self.extend_hidden([seq[b] for b in members], chunks)
            # Rows of h whose logits are needed, with their (row, target position).
            pick, where = [], []
            off = 0
            for b, n in zip(members, q_lens.tolist()):
                for j in range(n):
                    p = pos[b] + j
                    if p in need_sets[b]:
                        pick.append(off + j)
                        where.append((b, p + 1))
                off += n
                pos[b] += n
            for s0 in range(0, len(pick), max_logit_rows):
                sel = torch.tensor(pick[s0:s0 + max_logit_rows], device=h.device)
                tgt = [where[i] for i in range(s0, min(s0 + max_logit_rows, len(pick)))]
                bi = torch.tensor([t[0] for t in tgt])
                pi = torch.tensor([t[1] for t in tgt])
                nxt = ids[bi, pi].to(h.device)
                lp = self.sampler.token_logprobs(self.logits(h.index_select(0, sel)), nxt)
                out[bi.to(out.device), pi.to(out.device)] = lp.to(out.device)

    # -- rollout ----------------------------------------------------------------
    def generate(self, prompts, *, group_size: int = 1, max_new_tokens: int = 16,
                 sampling: SamplingConfig | None = None, force_tokens=None, first_id: int = 0,
                 release: bool = True, step_callback=None) -> dict:
        """Roll out ``group_size`` completions per prompt.

        Each prompt is prefilled once; the other members of its group fork the
        prompt's pages (copy-on-write) and start from the same next-token
        logits.  Returns ``{"sequence_ids", "tokens" (list per sequence),
        "logprobs" (list per sequence: the temperature-1 log-probability of
        each emitted token, the old-policy value of rollout.py:456-472),
        "argmax" (per token, the greedy token of the logits it was drawn
        from), "kv_pressure" (counters, below), "steps" (decode loop
        iterations)}``.  ``force_tokens[i]`` (optional) feeds sequence i those
        tokens instead of sampled ones (teacher forcing).

        KV pressure (continuous.py:875-937): before each step, sequences whose
        next token needs a free block (a block boundary, or a copy-on-write
        copy of a shared tail) are admitted only while free blocks remain, in
        order of how long they have waited; the others keep their pending
        logits for a later step (soft preemption, counted as the reference
        counts it).  When that would leave more than a quarter of the batch
        waiting (or nothing admitted), the newest sequences are evicted (their
        blocks released) and re-prefilled from their prompts and tokens once
        blocks are free again, so a pool too small for the whole batch
        finishes instead of raising.
        ``step_callback(sequence_ids, tokens, logprobs)``, if given, is called
        once per loop iteration with that iteration's sampled rows (device
        tensors; possibly none).
        """
        cfg = sampling or SamplingConfig()
        sampler = self.sampler
        sampler.reseed(cfg.seed)
        n_groups = len(prompts)
        heads = [first_id + g * group_size for g in range(n_groups)]
        marks = None
        if self.device.type == "cuda":
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            marks[0].record()
        logits = self.prefill(heads, prompts)
        if marks is not None:
            marks[1].record()
        seq_ids, next_logits = [], []
        for g in range(n_groups):
            for m in range(group_size):
                sid = heads[g] + m
                if m:
                    self.store.fork(heads[g], sid)
                seq_ids.append(sid)
                next_logits.append(logits[g])
        cur = torch.stack(next_logits)
        n = len(seq_ids)
        # Prompt blocks the group members share (copy-on-write) right after the forks.
        alloc = getattr(self.store, "allocator", None)
        shared_after_prefill = (alloc.shared_block_count, alloc.used_block_count) if alloc is not None else (0, 0)
        if self.cuda_graphs:
            self.reserve_tables(max(int(torch.as_tensor(p).numel()) for p in prompts) + max_new_tokens)
        tokens = [[] for _ in range(n)]
        logprobs = [[] for _ in range(n)]
        argmax = [[] for _ in range(n)]
        kv = {"paged_kv_preempted_sequences": 0.0, "paged_kv_max_preempted_sequences": 0.0,
              "scheduler_decode_growth_block_demand": 0.0, "scheduler_decode_growth_blocks_admitted": 0.0,
              "paged_kv_evicted_sequences": 0.0, "paged_kv_recomputed_tokens": 0.0}
        cur_rows = list(range(n))      # sequence index of each row of ``cur``
        held: dict[int, torch.Tensor] = {}   # deferred sequences' pending logits
        evicted: list[int] = []        # released sequences to re-prefill, oldest first
        waited = [0] * n
        iterations = 0
        while cur_rows or held or evicted:
            iterations += 1
            if evicted:
                self._restore_evicted(evicted, held, prompts, group_size, seq_ids, tokens, kv,
                                      resident=len(cur_rows) + len(held))
            candidates = cur_rows + sorted(held)
            admitted = self._admit(candidates, seq_ids, waited, kv)
            # Deferring most of the batch would leave the step's weight and KV reads serving a few
            # tokens: evict instead (the newest sequences first, so a group leaves together and its
            # shared prompt blocks free with its last member) until at most a quarter waits.
            while candidates and (not admitted or len(candidates) - len(admitted) > max(1, len(candidates) // 4)):
                victim = max(candidates)
                self.store.release(seq_ids[victim])
                if victim in held:
                    del held[victim]
                else:
                    pos = cur_rows.index(victim)
                    cur_rows.pop(pos)
                    cur = torch.cat([cur[:pos], cur[pos + 1:]])
                evicted.append(victim)
                kv["paged_kv_evicted_sequences"] += 1.0
                candidates = [i for i in candidates if i != victim]
                admitted = self._admit(candidates, seq_ids, waited, kv)
            if not admitted:
                # Everything was evicted: the next iteration restores the oldest, if it fits at all.
                if not self._fits_alone(evicted[0], prompts, group_size, tokens):
                    raise RuntimeError("the KV pool cannot hold a single sequence of this rollout")
                continue
            if admitted == cur_rows and not held:
                rows = cur
            else:
                pos = {i: j for j, i in enumerate(cur_rows)}
                if all(i in pos for i in admitted):
                    rows = cur.index_select(0, torch.tensor([pos[i] for i in admitted], device=cur.device))
                else:
                    rows = torch.stack([cur[pos[i]] if i in pos else held[i] for i in admitted])
                adm = set(admitted)
                for i in candidates:
                    if i not in adm and i in pos:
                        held[i] = cur[pos[i]]
                for i in admitted:
                    held.pop(i, None)
                deferred = len(candidates) - len(admitted)
                kv["paged_kv_preempted_sequences"] += float(deferred)
                kv["paged_kv_max_preempted_sequences"] = max(kv["paged_kv_max_preempted_sequences"], float(deferred))
            if len(admitted) != len(candidates):
                adm = set(admitted)
                for i in candidates:
                    waited[i] = 0 if i in adm else waited[i] + 1
            elif held or any(waited[i] for i in admitted):
                for i in admitted:
                    waited[i] = 0
            if force_tokens is not None:
                nxt = torch.tensor([int(force_tokens[i][len(tokens[i])]) for i in admitted], device=rows.device)
                _, _, am = sampler.sample(rows)
                chosen_lp = sampler.token_logprobs(rows, nxt)
            else:
                nxt, chosen_lp, am = sampler.sample(rows, cfg)
            if step_callback is not None:
                step_callback([seq_ids[i] for i in admitted], nxt, chosen_lp)
            nxt_h, lp_h, am_h = nxt.tolist(), chosen_lp.tolist(), am.tolist()
            still = []
            for j, i in enumerate(admitted):
                tokens[i].append(nxt_h[j])
                logprobs[i].append(lp_h[j])
                argmax[i].append(am_h[j])
                done = (self.eos_token_id is not None and nxt_h[j] == self.eos_token_id) or \
                    len(tokens[i]) >= max_new_tokens
                if not done:
                    still.append(j)
                elif release and self.store.has_sequence(seq_ids[i]):
                    self.store.release(seq_ids[i])
            cur_rows = [admitted[j] for j in still]
            if not still:
                cur = cur[:0]
                continue
            keep = torch.tensor(still, device=rows.device)
            eager = False
            if self.cuda_graphs:
                # A graphed step pads to a recorded batch size; placeholders may each take a block.
                free = getattr(self.store, "free_block_count", None)
                if free is not None:
                    k = len(cur_rows)
                    eager = free - self._growth_used < graph_batch(k) - k + 1
            cur = self.decode_step([seq_ids[i] for i in cur_rows], nxt[keep], eager=eager)
        if marks is not None:
            marks[2].record()
            marks[2].synchronize()
            self.last_timings = {
                "prefill_ms": marks[0].elapsed_time(marks[1]), "decode_ms": marks[1].elapsed_time(marks[2]),
                "prefill_tokens": sum(int(torch.as_tensor(p).numel()) for p in prompts),
                "decode_tokens": sum(len(t) for t in tokens),
                "shared_blocks_after_prefill": shared_after_prefill,
            }
        if release:
            for sid in seq_ids:
                if self.store.has_sequence(sid):
                    self.store.release(sid)
            self.release_placeholders()
        return {"sequence_ids": seq_ids, "tokens": tokens, "logprobs": logprobs, "argmax": argmax,
                "kv_pressure": kv, "steps": iterations}

    def _admit(self, candidates: list[int], seq_ids: list[int], waited: list[int], kv: dict) -> list[int]:
        """Growth admission (continuous.py:900-937, with copy-on-write copies counted as growth): the
        candidates whose next token fits the free blocks, longest-waiting first; in candidate order."""
        free = getattr(self.store, "free_block_count", None)
        self._growth_used = 0
        if free is None or free >= len(candidates):
            self._growth_used = len(candidates) if free is not None else 0
            return list(candidates)
        need = self.store.growth_blocks([seq_ids[i] for i in candidates])
        order = sorted(range(len(candidates)), key=lambda j: (-waited[candidates[j]], j))
        used, take = 0, []
        for j in order:
            if need[j] and used >= free:
                continue
            take.append(j)
            used += int(need[j])
        kv["scheduler_decode_growth_block_demand"] += float(need.sum())
        kv["scheduler_decode_growth_blocks_admitted"] += float(used)
        self._growth_used = used
        return [candidates[j] for j in sorted(take)]

    def _block_size(self) -> int:
        alloc = getattr(self.store, "allocator", None)
        return int(alloc.block_size_tokens) if alloc is not None else int(getattr(self.store, "block_size", 16))

    def _fits_alone(self, i: int, prompts, group_size: int, tokens: list) -> bool:
        n = int(torch.as_tensor(prompts[i // group_size]).numel()) + len(tokens[i])
        return int(self.store.free_block_count) >= -(-n // self._block_size()) + 1

    def _restore_evicted(self, evicted: list[int], held: dict, prompts, group_size: int, seq_ids: list[int],
                         tokens: list, kv: dict, resident: int) -> None:
        """Re-prefill evicted sequences, oldest first, while the free blocks cover them plus one block of
        growth for every resident sequence.  The evicted members of one GRPO group come back together:
        their prompt is prefilled once and forked (copy-on-write, as at the start of the rollout), then
        each member is extended by its own tokens; their next-token logits join the held rows."""
        bs = self._block_size()
        free = int(self.store.free_block_count)
        groups: dict[int, list[int]] = {}
        for i in evicted:
            groups.setdefault(i // group_size, []).append(i)
        plan, taken = [], 0
        for g, members in groups.items():
            plen = int(torch.as_tensor(prompts[g]).numel())
            need = -(-plen // bs)
            take = []
            for i in members:
                extra = -(-(plen + len(tokens[i])) // bs) - plen // bs + 1
                if free < need + extra + resident + taken + len(take) + 1:
                    break
                take.append(i)
                need += extra
            if not take:
                break
            plan.append((g, take))
            free -= need
            taken += len(take)
            if len(take) < len(members):
                break
        if not plan:
            return
        done = {i for _, take in plan for i in take}
        evicted[:] = [i for i in evicted if i not in done]
        prompt_logits = self.prefill([seq_ids[take[0]] for _, take in plan], [prompts[g] for g, _ in plan])
        kv["paged_kv_recomputed_tokens"] += float(sum(int(torch.as_tensor(prompts[g]).numel()) for g, _ in plan))
        members, chunks = [], []
        for j, (g, take) in enumerate(plan):
            for i in take:
                if i != take[0]:
                    self.store.fork(seq_ids[take[0]], seq_ids[i])
                if tokens[i]:
                    members.append(i)
                    chunks.append(torch.tensor(tokens[i], dtype=torch.long))
                else:
                    held[i] = prompt_logits[j]
        if members:
            logits = self._extend_chunked([seq_ids[i] for i in members], chunks)
            for j, i in enumerate(members):
                held[i] = logits[j]
                kv["paged_kv_recomputed_tokens"] += float(chunks[j].numel())

    def _extend_chunked(self, sequence_ids, chunks) -> torch.Tensor:
        """``extend`` in rounds of at most ``prefill_chunk_size`` tokens per sequence: logits of each
        chunk's last token [n, vocab]."""
        cs = self.prefill_chunk_size
        last = [None] * len(chunks)
        rounds = max((c.numel() + cs - 1) // cs for c in chunks)
        for r in range(rounds):
            sub = [j for j, c in enumerate(chunks) if c.numel() > r * cs]
            h, q_lens = self.extend_hidden([sequence_ids[j] for j in sub],
                                           [chunks[j][r * cs:(r + 1) * cs] for j in sub])
            ends = np.cumsum(q_lens) - 1
            for k, j in enumerate(sub):
                if (r + 1) * cs >= chunks[j].numel():
                    last[j] = h[int(ends[k])]
        return self.logits(torch.stack(last))


def _paged_cache_classes():
    """The HF ``Cache`` subclass (built on first use, so that importing this module needs no transformers)."""
    from transformers.cache_utils import Cache, CacheLayerMixin

    class PagedCacheLayer(CacheLayerMixin):
        """One decoder layer's view of a ``PagedCache``: its K/V live in the store's pages."""

        is_sliding = False
        is_compileable = False

        def __init__(self, cache, layer_idx: int) -> None:
            super().__init__()
            self._cache = cache
            self.layer_idx = layer_idx
            self.is_initialized = True

        def lazy_initialization(self, key_states, value_states) -> None:
            return None

        def update(self, key_states, value_states, *args, **kwargs):
            return self._cache._update(key_states, value_states, self.layer_idx)

        def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
            return self._cache._cached + query_length, 0

        def get_seq_length(self) -> int:
            return self._cache._cached

        def get_max_cache_shape(self) -> int:
            return -1

    class PagedCache(Cache):
        """An HF ``Cache`` whose K/V live in a ``PagedKVCacheStore``'s pages: batch row b is the store's
        sequence ``sequence_ids[b]`` (reserved beforehand, possibly with cached tokens).

        ``update`` -- HF's per-layer cache call (transformers cache_utils.py:102-120, called at
        modeling_qwen2.py:225) -- appends the step's tokens to every sequence (allocator, once per
        forward, at layer 0), writes the layer's new K/V into their pages (scatter kernel) and returns
        the layer's whole K/V [B, Hkv, T, D] gathered from the pages (gather kernel), so the model's
        own attention runs unchanged over exactly the values a ``DynamicCache`` would hold.  The
        batch's sequences must hold equal token counts (as a ``DynamicCache`` batch does: padding is
        in the attention mask).

        With ``kernels=True`` (the model switched to the ``paged_b200`` attention by
        ``use_paged_attention``) nothing is gathered: at layer 0 of each forward the cache lays out a
        decode step (one token per sequence) or a prefill of the batch's equal chunks, ``update``
        returns the fresh K/V, and the attention appends and attends through the store's kernels
        (fused append + paged decode, or the chunked-prefill kernel), for that forward's layers.
        """

        def __init__(self, store, sequence_ids, num_layers: int, kernels: bool = False) -> None:
            self.store = store
            self.kernels = bool(kernels)
            self.ids = np.ascontiguousarray(np.asarray(sequence_ids, dtype=np.int64).reshape(-1))
            counts = store.token_counts(self.ids) if self.ids.size else np.zeros(0, dtype=np.int64)
            if counts.size and (counts != counts[0]).any():
                raise ValueError("the sequences of a PagedCache batch must hold equal token counts")
            self._cached = int(counts[0]) if counts.size else 0
            self._num_layers = int(num_layers)
            self._new_slots = None
            self._all_slots = None
            super().__init__(layers=[PagedCacheLayer(self, i) for i in range(self._num_layers)])

        def _update(self, key_states, value_states, layer_idx: int):
            b, hkv, t, d = key_states.shape
            if b != self.ids.size:
                raise ValueError(f"batch of {b} rows for a PagedCache of {self.ids.size} sequences")
            store = self.store
            if self.kernels:
                # The model's paged_b200 attention appends and attends through the store's kernels.
                if layer_idx == 0:
                    store._ensure_pool(self._num_layers, hkv, d, key_states.dtype, key_states.device)
                    if t == 1:
                        ph = _Phase("decode", store, step=store.decode_step(self.ids))
                    else:
                        store.append_many(self.ids, np.full(self.ids.size, t, dtype=np.int64))
                        ph = _Phase("prefill", store, sequence_ids=self.ids.tolist(),
                                    q_lens=np.full(self.ids.size, t, dtype=np.int64))
                    self._cached += t
                    _local.cache_phase = ph
                    _local.cache_layers_left = self._num_layers
                return key_states, value_states
            if layer_idx == 0:
                pool = store._ensure_pool(self._num_layers, hkv, d, key_states.dtype, key_states.device)
                store.append_many(self.ids, np.full(self.ids.size, t, dtype=np.int64))
                self._cached += t
                # Slots of the new tokens (their blocks' fills recorded) and of every token.
                step = store.prefill_step(self.ids, np.full(self.ids.size, t, dtype=np.int64), hkv)
                self._new_slots = step.slots
                bs = pool.block_size
                tok = np.arange(self._cached, dtype=np.int64)
                rows = []
                for sid in self.ids.tolist():
                    blocks = np.asarray(store.allocator.view(sid).physical_blocks, dtype=np.int64)
                    rows.append(blocks[tok // bs] * bs + tok % bs)
                self._all_slots = torch.from_numpy(np.concatenate(rows)).to(pool.device)
            pool = store.pool
            k_new = key_states.permute(1, 0, 2, 3).reshape(hkv, b * t, d).contiguous()
            v_new = value_states.permute(1, 0, 2, 3).reshape(hkv, b * t, d).contiguous()
            pool.scatter(layer_idx, k_new.unsqueeze(0), v_new.unsqueeze(0), self._new_slots)
            n = self._cached
            keys = torch.empty((1, hkv, b * n, d), dtype=pool.dtype, device=pool.device)
            values = torch.empty_like(keys)
            pool.gather(layer_idx, keys, values, self._all_slots)
            return (keys[0].view(hkv, b, n, d).permute(1, 0, 2, 3),
                    values[0].view(hkv, b, n, d).permute(1, 0, 2, 3))

        def get_seq_length(self, layer_idx: int = 0) -> int:
            return self._cached

        def get_mask_sizes(self, query_length: int, layer_idx: int = 0) -> tuple[int, int]:
            return self._cached + query_length, 0

    PagedCache.__qualname__, PagedCacheLayer.__qualname__ = "PagedCache", "PagedCacheLayer"
    return PagedCache


_PAGED_CACHE_CLASS = None


def __getattr__(name: str):
    # ``PagedCache`` is a transformers ``Cache`` subclass, defined on first use so that importing
    # this module does not import transformers.
    global _PAGED_CACHE_CLASS
    if name == "PagedCache":
        if _PAGED_CACHE_CLASS is None:
            _PAGED_CACHE_CLASS = _paged_cache_classes()
        return _PAGED_CACHE_CLASS
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
