"""Load checkpoints by upstream (Hugging Face) tensor names, cut for this rank.

Names follow the upstream model families the engine serves:

* Kimi-delta attention layers (Kimi-Linear / GLM `linear_attention` naming), prefix
  ``model.layers.{i}.self_attn.``: ``q_proj k_proj v_proj`` ``[H*D, hid]``, ``f_a_proj g_a_proj``
  ``[D, hid]``, ``f_b_proj g_b_proj`` ``[H*D, D]``, ``b_proj`` ``[H, hid]``,
  ``{q,k,v}_conv1d.weight`` ``[H*D, 1, 4]``, ``A_log`` ``[H]``, ``dt_bias`` ``[H*D]``,
  ``o_norm.weight`` ``[D]``, ``o_proj`` ``[hid, H*D]``;
* sparse-MLA layers (DeepSeek-V3.2 naming): ``q_a_proj q_a_layernorm q_b_proj kv_a_proj_with_mqa
  kv_a_layernorm kv_b_proj o_proj`` and the indexer ``indexer.{wq_b, wk, k_norm, weights_proj}``;
  fp8 projections as ``weight`` (e4m3) + ``weight_scale_inv`` (one fp32 scale per 128 x 128 block);
* MLPs: ``mlp.{gate,up,down}_proj`` (dense), ``mlp.gate.weight`` (+ ``e_score_correction_bias``),
  ``mlp.experts.{e}.{gate,up,down}_proj.weight`` (bf16) or ``.{trellis,suh,svh}`` (EXL3),
  ``mlp.shared_experts.{gate,up,down}_proj``;
* ``model.embed_tokens.weight``, ``model.norm.weight``, ``lm_head.weight``,
  ``model.layers.{i}.{input,post_attention}_layernorm.weight``.

* Qwen3-Next-style layers: gated delta net under ``linear_attn.`` (``in_proj_qkvz`` grouped per key
  head as [q | k | v of its value heads | z of its value heads], ``in_proj_ba`` grouped the same way
  as [b | a], ``conv1d.weight`` over [q | k | v] channels, ``A_log``, ``dt_bias``, ``norm.weight``,
  ``out_proj``); gated attention under ``self_attn.`` (``q_proj`` per head [q | gate], ``k_proj``,
  ``v_proj``, ``q_norm``, ``k_norm``, ``o_proj``); ``mlp.shared_expert.*``;
* Engram layers: ``model.layers.{i}.engram.{kv, h_norm, k_norm}``; the n-gram embedding
  ``model.ple_proj.weight`` (the tables themselves are separate files).

Hybrid checkpoints (the reference's EXL3 + another method per module, vllm_sm80/kernels/exl3/hybrid.py:85):
``quantization_config.module_quantization = {"rules": [{"match": REGEX, "method": M}, ...], "default": M}``
gives each projection's method by the first rule whose regex searches its name: ``"exl3"`` (the module is
stored as ``{trellis, suh, svh}``) or ``"unquantized"`` / ``"fp8"`` (``weight`` [+ ``weight_scale_inv``]).
Routed experts load in the model's expert format; any other EXL3-stored projection is decoded at load
into the model's float weight (W = diag(suh) H W_trellis H diag(svh), exactly the EXL3 linear).  A module
no rule names is refused when there is no default.

Every load records which checkpoint tensors it consumed; ``load_hf(..., strict=True)`` refuses a
checkpoint with tensors nothing read (``LoadInventory``), so a misnamed or extra tensor cannot be
silently ignored.

Tensor-parallel cuts match the model's own (heads of q/k/v/b/conv/A_log/dt_bias, rows of q_b and
the per-head kv_b, columns of o_proj, intermediate columns of the experts in whole 128-column
blocks for EXL3, the vocab rows of lm_head); expert parallel keeps this rank's whole experts.  The
reference loads the same upstream names through vLLM's weight loaders
(vllm_sm80/models/glm5next/sm80_model.py:112, models/deepseek_v41/sm80_model.py:449).
Marlin-packed experts load from this package's own checkpoints (checkpoint.py), not from GPTQ files.
"""

from __future__ import annotations

import glob
import os
from collections.abc import Mapping

import torch

from .formats import exl3 as fx
from .formats import fp8 as f8
from .parallel import state as pstate


class MissingTensor(KeyError):
    pass


class UnusedTensors(ValueError):
    pass


# tensors a checkpoint may carry that no module of the engine reads (derived buffers, drafter heads the
# config does not enable)
_IGNORED = (".rotary_emb.inv_freq", "mlp.shared_expert_gate.weight", "mtp.", "model.mtp")


class _Tracked(Mapping):
    """A tensor mapping that records the names read from it (the load inventory)."""

    def __init__(self, base: Mapping, rules=None, codebook: int = 2):
        self.base, self.used = base, set()
        self.rules, self.codebook = rules, codebook

    def __getitem__(self, k):
        self.used.add(k)
        return self.base[k]

    def __contains__(self, k):
        return k in self.base

    def __iter__(self):
        return iter(self.base)

    def __len__(self):
        return len(self.base)

    def unused(self) -> list[str]:
        return sorted(k for k in self.base if k not in self.used and not any(i in k for i in _IGNORED))


def module_method(rules: dict | None, name: str) -> str | None:
    """The method a hybrid checkpoint's rules give module `name` (first regex match, else the default);
    None without rules.  Raises for a module no rule covers when there is no default."""
    import re

    if not rules:
        return None
    for r in rules.get("rules", []):
        if re.search(r["match"], name):
            return r["method"]
    if "default" in rules:
        return rules["default"]
    raise ValueError(f"hybrid checkpoint: no module_quantization rule matches {name} and there is no default")


def _exl3_dense(t: Mapping, name: str, codebook: int) -> torch.Tensor:
    """The dense [out, in] fp32 weight of an EXL3-stored projection: the EXL3 linear applied to the
    identity (diag(suh) H W H diag(svh), logical sizes from the stored vectors)."""
    tr, suh, svh = _get(t, name + ".trellis"), _get(t, name + ".suh"), _get(t, name + ".svh")
    bits_x2 = tr.shape[2] // 8
    m = fx.Exl3Matrix(tr, suh, svh, bits_x2, codebook, suh.shape[0], svh.shape[0])
    W = fx.decode_weight(tr, bits_x2, codebook).float()
    return fx.linear(torch.eye(suh.shape[0]), m, W).t().contiguous()


def open_dir(path: str, readahead: bool = False) -> Mapping[str, torch.Tensor]:
    """All tensors of the ``*.safetensors`` files of a directory, read lazily by name.  readahead:
    page the shards in on a background thread meanwhile.  With ``VLLM_B200_OVERRIDE`` (a sidecar
    manifest) and ``VLLM_B200_OVERRIDE_SHA256`` set, the manifest's tensors come from its sidecar
    (checkpoint_override.apply_override)."""
    from safetensors import safe_open

    from . import envs
    from .checkpoint_override import Readahead, apply_override

    handles = {}
    index = {}
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if readahead:
        Readahead(files).__enter__()  # daemon thread; nothing waits for it
    for f in files:
        h = safe_open(f, framework="pt")
        handles[f] = h
        for k in h.keys():
            index[k] = f

    class _Lazy(Mapping):
        def __getitem__(self, k):
            if k not in index:
                raise MissingTensor(k)
            return handles[index[k]].get_tensor(k)

        def __iter__(self):
            return iter(index)

        def __len__(self):
            return len(index)

    lazy = _Lazy()
    manifest = envs.get("VLLM_B200_OVERRIDE")
    if manifest:
        lazy, _names = apply_override(lazy, manifest, envs.get("VLLM_B200_OVERRIDE_SHA256"))
    return lazy


def _get(t: Mapping, name: str) -> torch.Tensor:
    if name not in t:
        raise MissingTensor(name)
    return t[name]


def _dense(t: Mapping, name: str) -> torch.Tensor:
    """A projection's weight as float: bf16 as stored, fp8 dequantised with its block scales, an EXL3-stored
    module (hybrid checkpoints) decoded."""
    rules = getattr(t, "rules", None)
    method = module_method(rules, name) if rules else None
    if method == "exl3" or (method is None and name + ".weight" not in t and name + ".trellis" in t):
        return _exl3_dense(t, name, getattr(t, "codebook", 2))
    w = _get(t, name + ".weight")
    if w.dtype == torch.float8_e4m3fn:
        return f8.dequantize(w, _get(t, name + ".weight_scale_inv").float())
    return w.float()


def _rows(x: torch.Tensor, tp: int, r: int) -> torch.Tensor:
    n = x.shape[0] // tp
    return x[r * n:(r + 1) * n]


def _cols(x: torch.Tensor, tp: int, r: int) -> torch.Tensor:
    n = x.shape[1] // tp
    return x[:, r * n:(r + 1) * n]


def _set(dst: torch.Tensor, src: torch.Tensor) -> None:
    if tuple(dst.shape) != tuple(src.shape):
        raise ValueError(f"shape {tuple(src.shape)} does not fit {tuple(dst.shape)}")
    with torch.no_grad():
        dst.copy_(src.to(dst.dtype))


def _set_linear(lin, w: torch.Tensor) -> None:
    """A bf16 Linear or an fp8 block-scaled projection (re-quantised from the dense weight)."""
    if hasattr(lin, "lin"):  # Fp8Proj
        q, s = f8.quantize(w.float().cpu())
        _set(lin.lin.weight, q.view(lin.lin.weight.dtype) if q.dtype != lin.lin.weight.dtype else q)
        _set(lin.lin.scale, s)
    else:
        _set(lin.weight, w)


def _load_kda(a, t, p, tp, r):
    H, D = a.H * tp, a.D
    q, k, v = (_rows(_dense(t, p + n), tp, r) for n in ("q_proj", "k_proj", "v_proj"))
    fa, ga = _dense(t, p + "f_a_proj"), _dense(t, p + "g_a_proj")
    b = _rows(_dense(t, p + "b_proj"), tp, r)
    w = torch.cat([q, k, v, fa, ga, b], 0)
    pad = a.in_proj.weight.shape[0] - w.shape[0]
    _set_linear(a.in_proj, torch.cat([w, w.new_zeros(pad, w.shape[1])], 0))
    _set_linear(a.f_b, _rows(_dense(t, p + "f_b_proj"), tp, r))
    _set_linear(a.g_b, _rows(_dense(t, p + "g_b_proj"), tp, r))
    conv = torch.stack([_get(t, p + f"{n}_conv1d.weight").float().reshape(H, D, 4) for n in ("q", "k", "v")])
    _set(a.conv_w, conv[:, r * a.H:(r + 1) * a.H].reshape(-1, 4))
    _set(a.a_log, _rows(_get(t, p + "A_log").float().reshape(H), tp, r))
    _set(a.g_bias, _rows(_get(t, p + "dt_bias").float().reshape(H * D), tp, r))
    _set(a.norm_w, _get(t, p + "o_norm.weight"))
    _set_linear(a.o_proj, _cols(_dense(t, p + "o_proj"), tp, r))


def _gdn_groups(cfg_kda, Hv_local, tp, r):
    """For this rank's value heads: (key head, index in its group) of each, and the group size."""
    Hv = cfg_kda.num_heads
    Hk = cfg_kda.num_k_heads or Hv
    rep = Hv // Hk
    heads = list(range(r * Hv_local, (r + 1) * Hv_local))
    return [(j // rep, j % rep) for j in heads], rep, Hk


def _load_gdn(a, t, p, tp, r, cfg):
    """Gated delta net from Qwen3-Next names (rows grouped per key head)."""
    D = a.D
    grp, rep, Hk = _gdn_groups(cfg.kda, a.H, tp, r)
    qkvz = _dense(t, p + "in_proj_qkvz").view(Hk, 2 * D + 2 * rep * D, -1)
    ba = _dense(t, p + "in_proj_ba").view(Hk, 2 * rep, -1)
    q = torch.cat([qkvz[h, :D] for h, _ in grp])
    k = torch.cat([qkvz[h, D:2 * D] for h, _ in grp])
    v = torch.cat([qkvz[h, 2 * D + i * D:2 * D + (i + 1) * D] for h, i in grp])
    z = torch.cat([qkvz[h, 2 * D + rep * D + i * D:2 * D + rep * D + (i + 1) * D] for h, i in grp])
    b = torch.stack([ba[h, i] for h, i in grp])
    av = torch.stack([ba[h, rep + i] for h, i in grp])
    w = torch.cat([q, k, v, z, b, av], 0)
    pad = a.in_proj.weight.shape[0] - w.shape[0]
    _set_linear(a.in_proj, torch.cat([w, w.new_zeros(pad, w.shape[1])], 0))
    conv = _get(t, p + "conv1d.weight").float().reshape(-1, 4)
    cq = torch.cat([conv[h * D:(h + 1) * D] for h, _ in grp])
    ck = torch.cat([conv[Hk * D + h * D:Hk * D + (h + 1) * D] for h, _ in grp])
    cv = torch.cat([conv[2 * Hk * D + (h * rep + i) * D:2 * Hk * D + (h * rep + i + 1) * D] for h, i in grp])
    _set(a.conv_w, torch.cat([cq, ck, cv], 0))
    _set(a.a_log, _rows(_get(t, p + "A_log").float(), tp, r))
    _set(a.dt_bias, _rows(_get(t, p + "dt_bias").float(), tp, r))
    _set(a.norm_w, _get(t, p + "norm.weight"))
    _set_linear(a.o_proj, _cols(_dense(t, p + "out_proj"), tp, r))


def _load_gqa(a, t, p, tp, r, cfg):
    """Gated attention from Qwen3-Next names; key-value heads cut or replicated as the model keeps them."""
    g = cfg.gqa
    hd = g.head_dim
    qg = _rows(_dense(t, p + "q_proj"), tp, r)
    if g.num_kv_heads % tp == 0:
        kv0 = r * (g.num_kv_heads // tp)
    else:
        kv0 = r // (tp // g.num_kv_heads)
    k = _dense(t, p + "k_proj")[kv0 * hd:(kv0 + a.nkv) * hd]
    v = _dense(t, p + "v_proj")[kv0 * hd:(kv0 + a.nkv) * hd]
    _set_linear(a.in_proj, torch.cat([qg, k, v], 0))
    _set(a.q_norm_w, _get(t, p + "q_norm.weight"))
    _set(a.k_norm_w, _get(t, p + "k_norm.weight"))
    _set_linear(a.o_proj, _cols(_dense(t, p + "o_proj"), tp, r))


def _load_engram(e, t, p):
    _set_linear(e.kv, _dense(t, p + "kv"))
    _set(e.h_norm_w, _get(t, p + "h_norm.weight"))
    _set(e.k_norm_w, _get(t, p + "k_norm.weight"))


def _load_mla(a, t, p, tp, r):
    m = a.m
    if getattr(a, "full_heads", False):  # every head on every rank (data-parallel attention)
        tp, r = 1, 0
    w = torch.cat([_dense(t, p + "q_a_proj"), _dense(t, p + "kv_a_proj_with_mqa"), _dense(t, p + "indexer.wk"),
                   _dense(t, p + "indexer.weights_proj")], 0)
    _set_linear(a.in_proj, w)
    _set(a.q_a_norm.weight, _get(t, p + "q_a_layernorm.weight"))
    _set(a.kv_a_norm_w, _get(t, p + "kv_a_layernorm.weight"))
    _set_linear(a.q_b, _rows(_dense(t, p + "q_b_proj"), tp, r))
    kvb = _rows(_dense(t, p + "kv_b_proj").view(m.num_heads, a.dn + a.dv, a.kvl), tp, r)
    _set(a.w_uk_t, kvb[:, :a.dn].transpose(1, 2))
    _set(a.w_uv_t, kvb[:, a.dn:])
    _set_linear(a.o_proj, _cols(_dense(t, p + "o_proj"), tp, r))
    _set_linear(a.idx_q, _dense(t, p + "indexer.wq_b"))
    _set(a.idx_k_ln_w, _get(t, p + "indexer.k_norm.weight"))
    if p + "indexer.k_norm.bias" in t:
        _set(a.idx_k_ln_b, _get(t, p + "indexer.k_norm.bias"))


def _load_dsa(a, t, p, tp, r):
    """DeepSeek-V4.1 attention under `attn.` (the reference's module names, models/deepseek_v41/
    sm80_attention.py:197-252): heads of wq_b and attn_sink and the wo_a groups cut by rank, wo_b by
    its input columns; the compressor and the indexer replicated."""
    _set_linear(a.wq_a, _dense(t, p + "wq_a"))
    _set(a.q_norm.weight, _get(t, p + "q_norm.weight"))
    _set_linear(a.wq_b, _rows(_dense(t, p + "wq_b"), tp, r))
    _set_linear(a.wkv, _dense(t, p + "wkv"))
    _set(a.kv_norm.weight, _get(t, p + "kv_norm.weight"))
    _set(a.sink, _rows(_get(t, p + "attn_sink").float(), tp, r))
    G, og, ig = a.wo_a.weight.shape
    _set(a.wo_a.weight, _rows(_dense(t, p + "wo_a").view(G * tp, og, ig), tp, r))
    _set_linear(a.wo_b, _cols(_dense(t, p + "wo_b"), tp, r))
    if a.ratio:
        _set(a.comp_norm, _get(t, p + "compressor.norm.weight"))
        w = _dense(t, p + "compressor.wkv")
        if a.ratio > 1:  # the compressor pools groups by gate scores: [wkv | wgate]
            w = torch.cat([w, _dense(t, p + "compressor.wgate")], 0)
        _set_linear(a.wkv_c, w)
        _set_linear(a.idx_q, _dense(t, p + "indexer.wq_b"))
        _set_linear(a.idx_w, _dense(t, p + "indexer.weights_proj"))
        _set(a.wk, _dense(t, p + "indexer.wk"))
        _set(a.k_norm, _get(t, p + "indexer.k_norm.weight"))


def _load_hc(hc, t, p):
    """One mHC boundary: `{p}_fn`, `{p}_scale`, `{p}_base` (the reference's hc_attn_* / hc_ffn_*
    names, models/deepseek_v41/sm80_model.py:159-161)."""
    _set(hc.fn, _get(t, p + "_fn"))
    _set(hc.scale, _get(t, p + "_scale"))
    _set(hc.base, _get(t, p + "_base"))


def _load_dense_mlp(mlp, t, p, tp, r):
    g, u = (_rows(_dense(t, p + n), tp, r) for n in ("gate_proj", "up_proj"))
    _set_linear(mlp.gate_up, torch.cat([g, u], 0))
    _set_linear(mlp.down, _cols(_dense(t, p + "down_proj"), tp, r))


def _expert_range(moe, E):
    emap = getattr(moe.experts, "expert_map", None)
    if emap is None:
        return list(range(E))
    emap = emap.cpu()
    return [int(e) for e in (emap >= 0).nonzero().flatten()]


def _load_moe(moe, t, p, tp, r):
    from .models.hybrid import BF16Experts
    from .ops.moe import Exl3Experts

    mc = moe.mc
    _set_linear(moe.gate, _dense(t, p + "gate"))
    if moe.e_bias is not None:
        _set(moe.e_bias, _get(t, p + "gate.e_score_correction_bias"))
    ep = getattr(moe.experts, "expert_map", None) is not None
    ttp, tr = (1, 0) if ep else (tp, r)
    experts = _expert_range(moe, mc.num_experts)
    ex = moe.experts
    if isinstance(ex, BF16Experts):
        for j, e in enumerate(experts):
            q = p + f"experts.{e}."
            g, u = (_rows(_dense(t, q + n), ttp, tr) for n in ("gate_proj", "up_proj"))
            _set(ex.gate_up[j], torch.cat([g, u], 0))
            _set(ex.down[j], _cols(_dense(t, q + "down_proj"), ttp, tr))
    elif isinstance(ex, Exl3Experts):
        mats = {w: [] for w in ("gate", "up", "down")}
        for e in experts:
            for w in mats:
                q = p + f"experts.{e}.{w}_proj."
                tr_, suh, svh = _get(t, q + "trellis"), _get(t, q + "suh"), _get(t, q + "svh")
                fin, fout = tr_.shape[0] * 16, tr_.shape[1] * 16
                mats[w].append(_cut_exl3(fx.Exl3Matrix(tr_, suh, svh, ex.bits_x2, ex.codebook, fin, fout), w,
                                         ttp, tr))
        new = Exl3Experts.from_matrices(mats["gate"], mats["up"], mats["down"], ex.expert_map, ex.swiglu_limit)
        for name in ("gate", "up", "down"):
            for part in ("trellis", "suh", "svh"):
                _set(getattr(ex, f"{name}_{part}"), getattr(new, f"{name}_{part}"))
    else:
        raise NotImplementedError("Marlin-packed experts load from this package's own checkpoints")
    if moe.shared is not None:
        rep = getattr(moe, "shared_replicated", False)  # expert parallel: the whole shared expert on every rank
        sp = p + ("shared_expert." if p + "shared_expert.gate_proj.weight" in t
                  or p + "shared_expert.gate_proj.trellis" in t else "shared_experts.")
        _load_dense_mlp(moe.shared, t, sp, 1 if rep else tp, 0 if rep else r)


def _cut_exl3(m: "fx.Exl3Matrix", which: str, tp: int, r: int) -> "fx.Exl3Matrix":
    """This rank's whole-H128 share of an expert matrix: intermediate columns of gate/up, rows of down."""
    if tp == 1:
        return m
    if which == "down":
        n = m.in_features // tp
        return fx.Exl3Matrix(m.trellis[r * n // 16:(r + 1) * n // 16].contiguous(), m.suh[r * n:(r + 1) * n].contiguous(),
                             m.svh, m.bits_x2, m.codebook, n, m.out_features)
    n = m.out_features // tp
    return fx.Exl3Matrix(m.trellis[:, r * n // 16:(r + 1) * n // 16].contiguous(), m.suh,
                         m.svh[r * n:(r + 1) * n].contiguous(), m.bits_x2, m.codebook, m.in_features, n)


def load_hf(model, tensors: Mapping[str, torch.Tensor] | str, strict: bool = False,
            quantization_config: dict | None = None) -> dict:
    """Fill a built HybridForCausalLM (this rank's stage and shards) from upstream-named tensors (a
    mapping, or a directory of safetensors files).  Returns the load inventory {"consumed": n, "unused":
    [names]}; with `strict` a checkpoint holding tensors nothing read is refused (UnusedTensors) -- on a
    single-stage, single-rank load, where every tensor has a reader.  `quantization_config` is the
    checkpoint's (hybrid `module_quantization` rules, EXL3 `codebook` marker)."""
    t = open_dir(tensors) if isinstance(tensors, str) else tensors
    qc = quantization_config or {}
    codebook = fx.MARKERS.get(qc.get("codebook", "mul1"), (2, 0))[0]
    t = _Tracked(t, qc.get("module_quantization"), codebook)
    cfg = model.cfg
    st = pstate.get()
    tp, r = st.tp_size, st.tp_rank
    if model.embed is not None:
        _set(model.embed, _get(t, "model.embed_tokens.weight"))
    if model.norm is not None:
        _set(model.norm.weight, _get(t, "model.norm.weight"))
    if model.lm_head is not None:
        _set_linear(model.lm_head, _rows(_dense(t, "lm_head"), tp, r))
    if getattr(model, "hc_head", None) is not None:
        _load_hc(model.hc_head, t, "model.hc_head")
    for layer in model.layers:
        p = f"model.layers.{layer.idx}."
        _set(layer.input_norm.weight, _get(t, p + "input_layernorm.weight"))
        _set(layer.post_norm.weight, _get(t, p + "post_attention_layernorm.weight"))
        if layer.kind == "dsa":
            _load_dsa(layer.attn, t, p + "attn.", tp, r)
        elif layer.kind == "gqa":
            _load_gqa(layer.attn, t, p + "self_attn.", tp, r, cfg)
        elif layer.kind == "kda" and cfg.kda.mode == "gdn":
            _load_gdn(layer.attn, t, p + "linear_attn.", tp, r, cfg)
        else:
            (_load_kda if layer.kind == "kda" else _load_mla)(layer.attn, t, p + "self_attn.", tp, r)
        if getattr(layer, "engram", None) is not None:
            _load_engram(layer.engram, t, p + "engram.")
        if getattr(layer, "hc_attn", None) is not None:
            _load_hc(layer.hc_attn, t, p + "hc_attn")
            if layer.hc_mlp is not None:
                _load_hc(layer.hc_mlp, t, p + "hc_ffn")
        if layer.mlp is None:
            continue
        if hasattr(layer.mlp, "gate_up"):
            _load_dense_mlp(layer.mlp, t, p + "mlp.", tp, r)
        else:
            _load_moe(layer.mlp, t, p + "mlp.", tp, r)
    if getattr(model, "ple", None) is not None:
        _set_linear(model.ple.proj, _dense(t, "model.ple_proj"))
    from .checkpoint import drop_decoded_caches

    drop_decoded_caches(model)
    unused = t.unused()
    if strict and unused:
        raise UnusedTensors(f"{len(unused)} checkpoint tensors have no reader, e.g. {unused[:5]}")
    return {"consumed": len(t.used), "unused": unused}


def export_hf(model) -> dict[str, torch.Tensor]:
    """The upstream-named tensors of a single-rank model (the inverse of `load_hf` at TP = 1)."""
    from .models.hybrid import BF16Experts
    from .ops.moe import Exl3Experts

    st = pstate.get()
    if st.tp_size != 1 or st.pp_size != 1:
        raise ValueError("export_hf writes a whole model: run it at TP = PP = 1")
    out: dict[str, torch.Tensor] = {}

    def dense(lin):
        if hasattr(lin, "lin"):
            return f8.dequantize(lin.lin.weight, lin.lin.scale.float()).to(torch.bfloat16)
        return lin.weight.detach()

    def put(name: str, lin) -> None:
        """A projection under `name`: fp8 stays fp8 (+ its block scales), bf16 as is."""
        if hasattr(lin, "lin"):
            out[name + ".weight"] = lin.lin.weight.detach()
            out[name + ".weight_scale_inv"] = lin.lin.scale.detach()
        else:
            out[name + ".weight"] = lin.weight.detach()

    out["model.embed_tokens.weight"] = model.embed.detach()
    if getattr(model, "hc_head", None) is not None:
        h = model.hc_head
        out["model.hc_head_fn"], out["model.hc_head_scale"], out["model.hc_head_base"] = (
            h.fn.detach(), h.scale.detach(), h.base.detach())
    out["model.norm.weight"] = model.norm.weight.detach()
    out["lm_head.weight"] = dense(model.lm_head)
    if getattr(model, "ple", None) is not None:
        out["model.ple_proj.weight"] = dense(model.ple.proj)
    for layer in model.layers:
        p = f"model.layers.{layer.idx}."
        out[p + "input_layernorm.weight"] = layer.input_norm.weight.detach()
        out[p + "post_attention_layernorm.weight"] = layer.post_norm.weight.detach()
        a = layer.attn
        q = p + "self_attn."
        for hc, n in ((getattr(layer, "hc_attn", None), "hc_attn"), (getattr(layer, "hc_mlp", None), "hc_ffn")):
            if hc is not None:
                out[p + n + "_fn"], out[p + n + "_scale"], out[p + n + "_base"] = (
                    hc.fn.detach(), hc.scale.detach(), hc.base.detach())
        if layer.kind == "dsa":
            q = p + "attn."
            out[q + "wq_a.weight"] = dense(a.wq_a)
            out[q + "q_norm.weight"] = a.q_norm.weight.detach()
            out[q + "wq_b.weight"] = dense(a.wq_b)
            out[q + "wkv.weight"] = dense(a.wkv)
            out[q + "kv_norm.weight"] = a.kv_norm.weight.detach()
            out[q + "attn_sink"] = a.sink.detach()
            out[q + "wo_a.weight"] = a.wo_a.weight.detach().reshape(-1, a.wo_a.weight.shape[-1])
            out[q + "wo_b.weight"] = dense(a.wo_b)
            if a.ratio:
                out[q + "compressor.norm.weight"] = a.comp_norm.detach()
                w = dense(a.wkv_c)
                if a.ratio > 1:
                    out[q + "compressor.wkv.weight"], out[q + "compressor.wgate.weight"] = (
                        x.contiguous() for x in w.chunk(2, 0))
                else:
                    out[q + "compressor.wkv.weight"] = w
                out[q + "indexer.wq_b.weight"] = dense(a.idx_q)
                out[q + "indexer.weights_proj.weight"] = dense(a.idx_w)
                out[q + "indexer.wk.weight"] = a.wk.detach()
                out[q + "indexer.k_norm.weight"] = a.k_norm.detach()
        elif layer.kind == "gqa":
            hd = model.cfg.gqa.head_dim
            w = dense(a.in_proj)
            nq = a.nh * 2 * hd
            out[q + "q_proj.weight"] = w[:nq].contiguous()
            out[q + "k_proj.weight"] = w[nq:nq + a.nkv * hd].contiguous()
            out[q + "v_proj.weight"] = w[nq + a.nkv * hd:nq + 2 * a.nkv * hd].contiguous()
            out[q + "q_norm.weight"] = a.q_norm_w.detach()
            out[q + "k_norm.weight"] = a.k_norm_w.detach()
            out[q + "o_proj.weight"] = dense(a.o_proj)
        elif layer.kind == "kda" and model.cfg.kda.mode == "gdn":
            q = p + "linear_attn."
            H, D = a.H, a.D
            grp, rep, Hk = _gdn_groups(model.cfg.kda, H, 1, 0)
            w = dense(a.in_proj)
            qs, ks, vs, zs = (w[i * H * D:(i + 1) * H * D].view(H, D, -1) for i in range(4))
            bs, as_ = w[4 * H * D:4 * H * D + H], w[4 * H * D + H:4 * H * D + 2 * H]
            rows, ba = [], []
            for h in range(Hk):
                js = [j for j, (hh, _) in enumerate(grp) if hh == h]
                rows += [qs[js[0]], ks[js[0]]] + [vs[j] for j in js] + [zs[j] for j in js]
                ba += [bs[j:j + 1] for j in js] + [as_[j:j + 1] for j in js]
            out[q + "in_proj_qkvz.weight"] = torch.cat(rows, 0).contiguous()
            out[q + "in_proj_ba.weight"] = torch.cat(ba, 0).contiguous()
            conv = a.conv_w.detach().view(3, H, D, 4)
            first = [next(j for j, (hh, _) in enumerate(grp) if hh == h) for h in range(Hk)]
            out[q + "conv1d.weight"] = torch.cat([conv[0, first].reshape(-1, 4), conv[1, first].reshape(-1, 4),
                                                  conv[2].reshape(-1, 4)], 0).unsqueeze(1).contiguous()
            out[q + "A_log"] = a.a_log.detach()
            out[q + "dt_bias"] = a.dt_bias.detach()
            out[q + "norm.weight"] = a.norm_w.detach()
            out[q + "out_proj.weight"] = dense(a.o_proj)
        elif layer.kind == "kda":
            H, D = a.H, a.D
            w = dense(a.in_proj)
            s = [H * D, H * D, H * D, D, D, H]
            parts = torch.split(w[:sum(s)], s, 0)
            for n, x in zip(("q_proj", "k_proj", "v_proj", "f_a_proj", "g_a_proj", "b_proj"), parts):
                out[q + n + ".weight"] = x.contiguous()
            out[q + "f_b_proj.weight"] = dense(a.f_b)
            out[q + "g_b_proj.weight"] = dense(a.g_b)
            conv = a.conv_w.detach().view(3, H * D, 1, 4)
            for i, n in enumerate("qkv"):
                out[q + f"{n}_conv1d.weight"] = conv[i].contiguous()
            out[q + "A_log"] = a.a_log.detach()
            out[q + "dt_bias"] = a.g_bias.detach()
            out[q + "o_norm.weight"] = a.norm_w.detach()
            out[q + "o_proj.weight"] = dense(a.o_proj)
        else:
            m = a.m
            w = dense(a.in_proj)
            s = [a.ql, a.kvl + a.dr, m.index_head_dim, m.index_n_heads]
            for n, x in zip(("q_a_proj", "kv_a_proj_with_mqa", "indexer.wk", "indexer.weights_proj"), torch.split(w, s, 0)):
                out[q + n + ".weight"] = x.contiguous()
            out[q + "q_a_layernorm.weight"] = a.q_a_norm.weight.detach()
            out[q + "kv_a_layernorm.weight"] = a.kv_a_norm_w.detach()
            put(q + "q_b_proj", a.q_b)
            out[q + "kv_b_proj.weight"] = torch.cat([a.w_uk_t.detach().transpose(1, 2), a.w_uv_t.detach()], 1).reshape(-1, a.kvl)
            put(q + "o_proj", a.o_proj)
            put(q + "indexer.wq_b", a.idx_q)
            out[q + "indexer.k_norm.weight"] = a.idx_k_ln_w.detach()
            out[q + "indexer.k_norm.bias"] = a.idx_k_ln_b.detach()
        if getattr(layer, "engram", None) is not None:
            e = layer.engram
            out[p + "engram.kv.weight"] = dense(e.kv)
            out[p + "engram.h_norm.weight"] = e.h_norm_w.detach()
            out[p + "engram.k_norm.weight"] = e.k_norm_w.detach()
        mlp = layer.mlp
        if mlp is None:
            continue
        q = p + "mlp."
        if hasattr(mlp, "gate_up"):
            g, u = dense(mlp.gate_up).chunk(2, 0)
            out[q + "gate_proj.weight"], out[q + "up_proj.weight"] = g.contiguous(), u.contiguous()
            out[q + "down_proj.weight"] = dense(mlp.down)
            continue
        out[q + "gate.weight"] = dense(mlp.gate)
        if mlp.e_bias is not None:
            out[q + "gate.e_score_correction_bias"] = mlp.e_bias.detach()
        ex = mlp.experts
        if isinstance(ex, BF16Experts):
            for e in range(ex.gate_up.shape[0]):
                g, u = ex.gate_up[e].detach().chunk(2, 0)
                out[q + f"experts.{e}.gate_proj.weight"] = g.contiguous()
                out[q + f"experts.{e}.up_proj.weight"] = u.contiguous()
                out[q + f"experts.{e}.down_proj.weight"] = ex.down[e].detach()
        elif isinstance(ex, Exl3Experts):
            for e in range(ex.num_local):
                for w in ("gate", "up", "down"):
                    for part in ("trellis", "suh", "svh"):
                        out[q + f"experts.{e}.{w}_proj.{part}"] = getattr(ex, f"{w}_{part}")[e].detach()
        else:
            raise NotImplementedError("Marlin-packed experts are exported by checkpoint.py")
        if mlp.shared is not None:
            g, u = dense(mlp.shared.gate_up).chunk(2, 0)
            out[q + "shared_experts.gate_proj.weight"] = g.contiguous()
            out[q + "shared_experts.up_proj.weight"] = u.contiguous()
            out[q + "shared_experts.down_proj.weight"] = dense(mlp.shared.down)
    return out
