"""Lightning-style PTH export of the hybrid teacher and TimeMix splicing.

Two offline tools for an external C++ inference engine (reference ``convert_qwen2rwkv_lightning.py:1-432``
and ``replace_timemix_lightning.py:1-363``):

* ``convert_hf``: a local Qwen3.5-family hybrid safetensors checkpoint -> one uncompressed ``.pth``
  state dict in the "rwkv_lightning_qwen_hybrid_v1" naming (``emb``, ``blocks.<i>.{ln1,ln2,att,ffn}``,
  ``ln_out``, ``head``) plus ``.config.json`` (geometry, runtime contract) and ``.manifest.json``
  (one entry per exported tensor) sidecars. Only names and storage layout change: GDN ``in_proj_qkv`` is
  split into receptance/key/value rows, the per-head packed ``q_proj`` [Q_h, gate_h] rows are split into
  receptance and gate, conv1d weights lose their singleton axis; no transposes, no dtype casts.
* ``splice_timemix``: replaces the attention tensors of chosen blocks of such a PTH with trained TimeMix
  weights read from ``migrated.safetensors`` snapshots (``<layer>.<param>`` keys; files in natural path
  order, later files win), LoRA factors transposed to [out, in], [1, 1, C] vectors flattened. Head size
  per layer is inferred from ``r_k``.

Both write to a temporary file in the output directory, check the zip structure (stored, not
compressed), optionally re-read every tensor bitwise, write the sidecars atomically and only then
rename the PTH into place. The tensor names, sidecar keys and contract strings are the file format the
engine reads; they are kept identical to the reference's.
"""
import hashlib
import json
import math
import os
import re
import shutil
import tempfile
import zipfile
from collections import Counter, defaultdict
from dataclasses import dataclass
from datetime import datetime, timezone
from pathlib import Path

import torch
from safetensors import safe_open

FORMAT = "rwkv_lightning_qwen_hybrid_v1"
TIMEMIX_KIND = "rwkv7_timemix"
FLOAT_BYTES = {"BF16": 2, "F16": 2, "F32": 4}
LOW_RANK = frozenset({"w1", "w2", "a1", "a2", "g1", "g2"})
_CHUNK = 32 << 20


def _bar(total, desc, quiet, **kw):
    from tqdm.auto import tqdm
    return tqdm(total=total, desc=desc, disable=quiet, **kw)


def sidecar(path, kind):
    return Path(path).with_suffix(f".{kind}.json")


def atomic_json(path, value):
    """Write `value` as indented JSON next to `path`, flush it to disk, then rename it over `path`."""
    path = Path(path)
    text = json.dumps(value, indent=2, ensure_ascii=False) + "\n"
    fd, partial = tempfile.mkstemp(prefix=path.name + ".", suffix=".partial", dir=path.parent)
    try:
        os.write(fd, text.encode("utf-8"))
        os.fsync(fd)
    finally:
        os.close(fd)
    try:
        os.replace(partial, path)
    except BaseException:
        Path(partial).unlink(missing_ok=True)
        raise


# ---------------------------------------------------------------- HF checkpoint -> PTH
_GEOMETRY_KEYS = ("hidden_size", "intermediate_size", "num_hidden_layers", "vocab_size", "linear_num_key_heads",
                  "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim", "linear_conv_kernel_dim",
                  "num_attention_heads", "num_key_value_heads", "head_dim")
_LAYER_KINDS = {"linear_attention", "full_attention"}


def _layer_kinds(text, layers):
    """``layer_types``, or the pattern ``full_attention_interval`` implies (every n-th block full attention)."""
    if text.get("layer_types") is not None:
        return list(text["layer_types"])
    interval = int(text["full_attention_interval"])
    if interval < 1:
        raise ValueError(f"full_attention_interval must be at least 1, got {interval}")
    return ["full_attention" if index % interval == interval - 1 else "linear_attention" for index in range(layers)]


def geometry(config):
    """Validated text-model geometry of a Qwen3.5-family hybrid config.json."""
    text = config.get("text_config", config)
    if text.get("quantization_config") or config.get("quantization_config"):
        raise ValueError("quantized checkpoints (FP8, INT4, ...) are not accepted; convert the BF16/FP16/FP32 release")
    if text.get("model_type") not in ("qwen3_5", "qwen3_5_text"):
        raise ValueError(f"model_type {text.get('model_type')!r} is not a Qwen3.5 text model")
    g = {key: int(text[key]) for key in _GEOMETRY_KEYS}
    bad = [key for key, value in g.items() if value < 1]
    if bad:
        raise ValueError(f"non-positive model dimensions: {bad}")
    kinds = _layer_kinds(text, g["num_hidden_layers"])
    rules = (
        (len(kinds) == g["num_hidden_layers"] and set(kinds) <= _LAYER_KINDS,
         "layer_types must name one block per layer, each linear_attention (GDN) or full_attention"),
        (text.get("hidden_act", "silu") in ("silu", "swish"), "the MLP must be SiLU-gated (SwiGLU)"),
        (g["linear_num_value_heads"] % g["linear_num_key_heads"] == 0,
         "GDN value heads must be a multiple of its key heads"),
        (g["num_attention_heads"] % g["num_key_value_heads"] == 0,
         "attention heads must be a multiple of the KV heads"),
        (g["linear_key_head_dim"] == g["linear_value_head_dim"],
         "GDN key and value head sizes must be equal (square recurrent state)"),
        (text.get("attn_output_gate", True) is True, "full attention must carry the sigmoid output gate"),
    )
    for holds, message in rules:
        if not holds:
            raise ValueError(message)
    g["layer_types"] = kinds
    g["key_dim"] = g["linear_num_key_heads"] * g["linear_key_head_dim"]
    g["value_dim"] = g["linear_num_value_heads"] * g["linear_value_head_dim"]
    g["attention_bias"] = bool(text.get("attention_bias", False))
    g["tie_word_embeddings"] = bool(text.get("tie_word_embeddings", config.get("tie_word_embeddings", False)))
    return g


def checkpoint_index(src):
    """tensor name -> shard file name, from the index or by scanning the shards."""
    src = Path(src)
    index = src / "model.safetensors.index.json"
    if index.is_file():
        names = json.loads(index.read_text())["weight_map"]
    else:
        names = {}
        shards = sorted(src.glob("*.safetensors"))
        if not shards:
            raise FileNotFoundError(f"No safetensors checkpoint in {src}")
        for shard in shards:
            with safe_open(str(shard), framework="pt", device="cpu") as f:
                for key in f.keys():
                    if key in names:
                        raise ValueError(f"Duplicate input tensor: {key}")
                    names[key] = shard.name
    if not names:
        raise ValueError("Empty checkpoint index.")
    for rel in set(names.values()):
        if Path(rel).is_absolute() or ".." in Path(rel).parts:
            raise ValueError(f"Unsafe shard path in index: {rel}")
        if not (src / rel).is_file():
            raise FileNotFoundError(f"Missing shard: {src / rel}")
    return names


@dataclass(frozen=True)
class Mapping:
    source: str
    targets: tuple
    shape: tuple
    op: str = "copy"


def plan(keys, g):
    """Mapping of every text tensor; unmapped text tensors are an error, never dropped silently."""
    roots = [r for r in ("model.language_model.", "language_model.", "model.") if r + "embed_tokens.weight" in keys]
    if len(roots) != 1:
        raise ValueError(f"Cannot uniquely identify the text backbone: {roots}")
    root = roots[0]
    C, F, V = g["hidden_size"], g["intermediate_size"], g["vocab_size"]
    kd, vd, hv, dv = g["key_dim"], g["value_dim"], g["linear_num_value_heads"], g["linear_value_head_dim"]
    qd, kvd, hd = g["num_attention_heads"] * g["head_dim"], g["num_key_value_heads"] * g["head_dim"], g["head_dim"]
    out = []

    def need(source, targets, shape, op="copy"):
        if source not in keys:
            raise ValueError(f"Missing required source tensor: {source}")
        out.append(Mapping(source, (targets,) if isinstance(targets, str) else tuple(targets), tuple(shape), op))

    need(root + "embed_tokens.weight", "emb.weight", (V, C))
    need(root + "norm.weight", "ln_out.weight", (C,))
    heads = [k for k in ("lm_head.weight", "model.lm_head.weight", "language_model.lm_head.weight") if k in keys]
    if len(heads) > 1:
        raise ValueError(f"Ambiguous LM head: {heads}")
    if heads:
        need(heads[0], "head.weight", (V, C))
    elif not g["tie_word_embeddings"]:
        raise ValueError("Untied model is missing lm_head.weight.")
    for i, kind in enumerate(g["layer_types"]):
        src, dst = f"{root}layers.{i}.", f"blocks.{i}."
        need(src + "input_layernorm.weight", dst + "ln1.weight", (C,))
        need(src + "post_attention_layernorm.weight", dst + "ln2.weight", (C,))
        need(src + "mlp.up_proj.weight", dst + "ffn.key.weight", (F, C))
        need(src + "mlp.down_proj.weight", dst + "ffn.value.weight", (C, F))
        need(src + "mlp.gate_proj.weight", dst + "ffn.gate.weight", (F, C))
        att = dst + "att."
        if kind == "linear_attention":
            p = src + "linear_attn."
            need(p + "in_proj_qkv.weight", [att + n + ".weight" for n in ("receptance", "key", "value")],
                 (2 * kd + vd, C), "split_qkv")
            for s, t, shape in (("in_proj_z.weight", "gate.weight", (vd, C)),
                                ("in_proj_a.weight", "decay.weight", (hv, C)),
                                ("in_proj_b.weight", "beta.weight", (hv, C)),
                                ("A_log", "A_log", (hv,)), ("dt_bias", "dt_bias", (hv,)),
                                ("norm.weight", "ln_x.weight", (dv,)), ("out_proj.weight", "output.weight", (C, vd))):
                need(p + s, att + t, shape)
            need(p + "conv1d.weight", att + "conv1d.weight", (2 * kd + vd, 1, g["linear_conv_kernel_dim"]),
                 "squeeze_conv")
            if p + "conv1d.bias" in keys:
                need(p + "conv1d.bias", att + "conv1d.bias", (2 * kd + vd,))
        else:
            p = src + "self_attn."
            need(p + "q_proj.weight", (att + "receptance.weight", att + "gate.weight"), (2 * qd, C), "split_q_gate")
            for s, t, shape in (("k_proj.weight", "key.weight", (kvd, C)), ("v_proj.weight", "value.weight", (kvd, C)),
                                ("o_proj.weight", "output.weight", (C, qd)), ("q_norm.weight", "q_norm.weight", (hd,)),
                                ("k_norm.weight", "k_norm.weight", (hd,))):
                need(p + s, att + t, shape)
            if g["attention_bias"]:
                need(p + "q_proj.bias", (att + "receptance.bias", att + "gate.bias"), (2 * qd,), "split_q_gate")
                for s, t, n in (("k_proj", "key", kvd), ("v_proj", "value", kvd), ("o_proj", "output", C)):
                    need(p + s + ".bias", att + t + ".bias", (n,))
    used = {m.source for m in out}
    stray = sorted(k for k in keys if k.startswith(root) and k not in used)
    if stray:
        raise ValueError("Unmapped TEXT tensors (not silently dropped):\n" + "\n".join(stray[:30]))
    targets = [t for m in out for t in m.targets]
    if len(targets) != len(set(targets)):
        raise ValueError("Destination tensor-name collision.")
    return out, root, not heads


def apply(m, x, g):
    if tuple(x.shape) != m.shape:
        raise ValueError(f"Shape mismatch: {m.source}: {tuple(x.shape)} != {m.shape}")
    if m.op == "split_qkv":
        parts = x.split((g["key_dim"], g["key_dim"], g["value_dim"]), dim=0)
    elif m.op == "split_q_gate":  # rows are packed per head as [Q_h ; gate_h]
        rest = tuple(x.shape[1:])
        packed = x.reshape(g["num_attention_heads"], 2, g["head_dim"], *rest)
        parts = (packed[:, 0].reshape(-1, *rest), packed[:, 1].reshape(-1, *rest))
    elif m.op == "squeeze_conv":
        parts = (x[:, 0],)
    else:
        parts = (x,)
    return tuple(p.contiguous() for p in parts)


def _save_pth(state, out, quiet, verify):
    """torch.save into a temp file beside `out` (uncompressed zip), optional bitwise re-read; returns temp path."""
    fd, tmp = tempfile.mkstemp(prefix=out.stem + ".", suffix=".partial", dir=out.parent)
    try:
        with os.fdopen(fd, "wb") as f:
            torch.save(state, f, pickle_protocol=2, _use_new_zipfile_serialization=True)
            f.flush()
            os.fsync(f.fileno())
        with zipfile.ZipFile(tmp) as z:
            if not any(n.endswith("/data.pkl") for n in z.namelist()):
                raise ValueError("Saved PTH lacks data.pkl")
            if any(info.compress_type != zipfile.ZIP_STORED for info in z.infolist()):
                raise ValueError("Saved PTH contains compressed storages")
        if verify:
            _verify(Path(tmp), state, quiet)
        return tmp
    except BaseException:
        os.unlink(tmp)
        raise


def _verify(path, expected, quiet):
    loaded = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    if set(loaded) != set(expected):
        raise ValueError("Saved checkpoint tensor keys differ")
    total = sum(t.numel() * t.element_size() for t in expected.values())
    with _bar(total, "Verify bytes", quiet, unit="B", unit_scale=True) as bar:
        for name, want in expected.items():
            got = loaded[name]
            if got.dtype != want.dtype or got.shape != want.shape:
                raise ValueError(f"Saved tensor metadata differs: {name}")
            a = want.contiguous().view(torch.uint8).reshape(-1)
            b = got.contiguous().view(torch.uint8).reshape(-1)
            for lo in range(0, a.numel(), _CHUNK):  # bitwise: keeps signed zeros and NaN payloads exact
                hi = min(lo + _CHUNK, a.numel())
                if not torch.equal(a[lo:hi], b[lo:hi]):
                    raise ValueError(f"Saved tensor bytes differ: {name}, byte {lo}")
                bar.update(hi - lo)


def contract(tc):
    """Runtime contract recorded for the engine (format data: names and wording are part of the format)."""
    return {
        "checkpoint_linear_layout": "out_in_row_major", "dtype_policy": "preserve_source_dtype_and_bits",
        "plain_state_dict": True, "pickle_protocol": 2,
        "norm_weights": "raw_Qwen: 1+weight for ln1/ln2/ln_out/q_norm/k_norm",
        "gdn_output_norm": "ordinary_weight_RMSNorm_then_SiLU_gate",
        "norm_epsilon": float(tc.get("rms_norm_eps", 1e-6)),
        "gdn_qk_normalization": "x * rsqrt(sum(x*x) + 1e-6)", "gdn_state_layout": "B,Hv,K,V",
        "recommended_reference_state_dtype": "float32",
        "wkv_decay_input": "g = -exp(A_log) * softplus(decay_projection + dt_bias)",
        "wkv_decay_operation": "exp(g), NO clamp/sigmoid/exp(-exp(w))",
        "wkv_inputs": "r=q/sqrt(Dk), w=g, k=k, v=beta*v, a=k, b=-exp(g)*beta*k",
        "gdn_head_mapping": "hk = hv // (Hv / Hk); no weight-head duplication",
        "conv_layout": "packed_Q_K_V_channels,kernel; oldest_to_newest_tap_order",
        "attention": "source full GQA + Q/K norms + RoPE + sigmoid output gate; KV cache retained",
        "attention_q_gate_split": "source.view(Hq,2,Dh,C)[:,0/1]; reversible row split",
        "ffn": "value(silu(gate(x))*key(x)); NO ReLU-squared or time shift",
        "embedding": "direct embedding lookup; NO RWKV ln0 preprocessing",
    }


def convert_hf(src, dst, *, verify=False, dry_run=False, overwrite=False, quiet=False):
    src, dst = Path(src).expanduser().resolve(), Path(dst).expanduser().resolve()
    if dst.suffix != ".pth":
        raise ValueError("Output filename must end with .pth")
    config_path = src / "config.json"
    config = json.loads(config_path.read_text())
    g = geometry(config)
    where = checkpoint_index(src)
    mappings, root, tied = plan(set(where), g)
    outputs = (dst, sidecar(dst, "config"), sidecar(dst, "manifest"))
    if not dry_run and not overwrite:
        for path in outputs:
            if path.exists():
                raise FileExistsError(f"Already exists: {path}; use --overwrite explicitly.")
    by_shard = defaultdict(list)
    for m in mappings:
        by_shard[where[m.source]].append(m)
    nbytes, dtypes = 0, Counter()
    for shard, group in sorted(by_shard.items()):  # headers only: shapes and dtypes before any copy
        with safe_open(str(src / shard), framework="pt", device="cpu") as f:
            for m in group:
                info = f.get_slice(m.source)
                shape, dtype = tuple(info.get_shape()), info.get_dtype()
                if shape != m.shape or dtype not in FLOAT_BYTES:
                    raise ValueError(f"Unsupported tensor: {m.source}: {shape}, {dtype}; expected {m.shape}")
                nbytes += math.prod(shape) * FLOAT_BYTES[dtype]
                dtypes[dtype] += 1
    summary = {"source": str(src), "output": str(dst), "source_tensors": len(mappings),
               "output_tensors": sum(len(m.targets) for m in mappings) + int(tied), "source_tensor_bytes": nbytes,
               "dtypes": dict(dtypes), "layer_counts": dict(Counter(g["layer_types"])),
               "dropped_non_text_tensors": len(where) - len(mappings)}
    print(json.dumps(summary, ensure_ascii=False, indent=2), flush=True)
    if dry_run:
        return summary
    dst.parent.mkdir(parents=True, exist_ok=True)
    if shutil.disk_usage(dst.parent).free < nbytes + (256 << 20):
        raise OSError("Insufficient free disk space for a new PTH (old output is not removed first).")
    state, entries = {}, []
    with _bar(len(mappings), "Map weights", quiet, unit="tensor") as bar:
        for shard, group in sorted(by_shard.items()):
            with safe_open(str(src / shard), framework="pt", device="cpu") as f:
                for m in group:
                    for name, value in zip(m.targets, apply(m, f.get_tensor(m.source), g), strict=True):
                        state[name] = value
                        entries.append({"source": m.source, "shard": shard, "target": name, "transform": m.op,
                                        "shape": list(value.shape),
                                        "dtype": str(value.dtype).removeprefix("torch."),
                                        "source_shape": list(m.shape)})
                    bar.update(1)
    if tied:
        state["head.weight"] = state["emb.weight"]
        entries.append({"source": root + "embed_tokens.weight", "target": "head.weight",
                        "transform": "tied_embedding_alias", "shape": list(state["head.weight"].shape),
                        "dtype": str(state["head.weight"].dtype).removeprefix("torch.")})
    tmp = _save_pth(state, dst, quiet, verify)
    try:
        tc = config.get("text_config", config)
        meta = {"format": FORMAT, "requires_hybrid_backend": True, "weights_file": dst.name,
                "weights_bytes": os.path.getsize(tmp), "exported_utc": datetime.now(timezone.utc).isoformat(),
                "source_dir": str(src), "source_tensor_prefix": root,
                "source_config_sha256": hashlib.sha256(config_path.read_bytes()).hexdigest(),
                "source_config": config, "geometry": g, "summary": summary,
                "contract": contract(tc) | {"tokenizer_source_dir": str(src)}}
        atomic_json(sidecar(dst, "config"), meta)
        atomic_json(sidecar(dst, "manifest"), {"format": FORMAT, "tensors": entries,
                                               "dropped_non_text_keys": sorted(set(where) - {m.source
                                                                                             for m in mappings})})
        os.replace(tmp, dst)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)
    print(f"Saved: {dst}\nConfig: {sidecar(dst, 'config')}\nManifest: {sidecar(dst, 'manifest')}", flush=True)
    return summary


# ---------------------------------------------------------------- TimeMix splice
def export_tensor(name, value):
    """TimeMix parameter in the engine layout: matrices [out, in], broadcast vectors flat [C]."""
    if name in LOW_RANK:
        return value.T.contiguous()
    if value.ndim == 3 and tuple(value.shape[:2]) == (1, 1):
        return value.reshape(-1).contiguous()
    return value.contiguous()


def parse_layers(text):
    try:
        layers = [int(part) for part in text.split(",")]
    except ValueError as err:
        raise ValueError("--layers must be comma-separated integer layer indices") from err
    _check_layers(layers)
    return layers


def _check_layers(layers):
    if not layers or min(layers) < 0 or len(set(layers)) != len(layers):
        raise ValueError("layers must be distinct nonnegative indices")


def _natural(path):
    return [int(p) if p.isdigit() else p.lower() for p in re.split(r"(\d+)", path.as_posix())]


def timemix_shapes(width, layer, depth, head_size):
    from ..models.timemix import TimeMix
    with torch.device("meta"):
        core = TimeMix(width, layer, depth, head_size=head_size, backend="reference")
    return {k: tuple(v.shape) for k, v in core.state_dict().items()}


def scan_snapshots(weights, layers, width, depth, head_size=None):
    """Pick, per (layer, param), the last snapshot file holding it; infer and check each layer's geometry."""
    weights = Path(weights)
    files = [weights] if weights.is_file() else sorted(weights.rglob("*.safetensors"),
                                                        key=lambda p: _natural(p.relative_to(weights)))
    if not files:
        raise FileNotFoundError(f"No .safetensors files in {weights}")
    pick, shape_of, superseded = {}, {}, 0
    for path in files:
        with safe_open(str(path), framework="pt", device="cpu") as f:
            for key in f.keys():
                hit = re.fullmatch(r"(\d+)\.(.+)", key)
                if hit is None:
                    raise ValueError(f"Unexpected Theseus tensor key in {path}: {key}")
                layer, name = int(hit[1]), hit[2]
                if layer not in layers:
                    continue
                part = f.get_slice(key)
                if part.get_dtype() not in FLOAT_BYTES:
                    raise ValueError(f"Invalid tensor dtype {path}:{key}: {part.get_dtype()}")
                superseded += (layer, name) in pick
                pick[layer, name] = path
                shape_of[layer, name] = tuple(part.get_shape())
    sizes, schemas = {}, {}
    for layer in layers:
        rk = shape_of.get((layer, "r_k"))  # [heads, head size]: the only tensor that states the head size
        if rk is None:
            raise ValueError(f"Layer {layer} is incomplete: it has no r_k, so its head size is unknown")
        heads_ok = len(rk) == 2 and rk[0] * rk[1] == width
        if not heads_ok or rk[1] not in (64, 128):
            raise ValueError(f"Layer {layer}: r_k of shape {tuple(rk)} is not [width / D, D] with D 64 or 128")
        if head_size is not None and rk[1] != head_size:
            raise ValueError(f"Layer {layer} was trained with head_size={rk[1]}, but --head-size={head_size}; "
                             "this option validates, it does not reshape heads")
        sizes[layer] = rk[1]
        schemas[layer] = timemix_shapes(width, layer, depth, rk[1])
        have = {n for (i, n) in pick if i == layer}
        missing, unknown = schemas[layer].keys() - have, have - schemas[layer].keys()
        if missing:
            raise ValueError(f"Layer {layer} is incomplete; missing: {', '.join(sorted(missing))}")
        if unknown:
            raise ValueError(f"Unknown TimeMix parameters in layer {layer}: {', '.join(sorted(unknown))}")
        for name, shape in schemas[layer].items():
            if shape_of[layer, name] != shape:
                raise ValueError(f"Invalid tensor {pick[layer, name]}:{layer}.{name}: {shape_of[layer, name]} != "
                                 f"{shape}")
    return files, pick, superseded, schemas, sizes


def splice_timemix(base, weights, out, layers, *, head_size=None, dtype="base", dry_run=False, verify=False,
                   overwrite=False, quiet=False):
    base, weights, out = (Path(p).expanduser().resolve() for p in (base, weights, out))
    if not base.is_file() or not weights.exists():
        raise FileNotFoundError("--base must be a PTH file and --weights-dir a directory or safetensors file")
    if base == out or out.suffix != ".pth":
        raise ValueError("--out must be a new .pth path distinct from --base")
    _check_layers(layers)
    if head_size not in (None, 64, 128):
        raise ValueError("Invalid geometry or head_size")
    cfg_path, man_path = sidecar(base, "config"), sidecar(base, "manifest")
    if not cfg_path.is_file() or not man_path.is_file():
        raise FileNotFoundError("The base PTH needs its .config.json and .manifest.json sidecars")
    config, manifest = json.loads(cfg_path.read_text()), json.loads(man_path.read_text())
    if config.get("format") != FORMAT or manifest.get("format") != config["format"]:
        raise ValueError("Unsupported or inconsistent converted PTH metadata")
    if config.get("weights_file") != base.name:
        raise ValueError("Base config weights_file does not match --base")
    geo = config["geometry"]
    kinds = geo["layer_types"]
    width, depth = int(geo["hidden_size"]), int(geo["num_hidden_layers"])
    if len(kinds) != depth or width <= 0:
        raise ValueError("Invalid geometry or head_size")
    for layer in layers:
        if layer >= depth or kinds[layer] not in ("full_attention", "linear_attention", TIMEMIX_KIND):
            raise ValueError(f"Layer {layer} is not a replaceable mixer layer")
    files, pick, superseded, schemas, sizes = scan_snapshots(weights, layers, width, depth, head_size)
    print(json.dumps({"base": str(base), "output": str(out), "layers": layers, "head_sizes": sizes,
                      "wkv_kernel": "shared_dplr_fp32_v1", "safetensors_files": len(files),
                      "selected_tensors": len(pick), "superseded_tensor_versions": superseded}), flush=True)
    state = torch.load(base, map_location="cpu", weights_only=True, mmap=True)
    if not isinstance(state, dict) or "emb.weight" not in state:
        raise ValueError("Base PTH is not a converted model state_dict")
    base_dtype = state["emb.weight"].dtype
    if base_dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError(f"Unsupported base dtype: {base_dtype}")
    stale = []
    for layer in layers:
        found = [k for k in state if k.startswith(f"blocks.{layer}.att.")]
        if not found:
            raise ValueError(f"Base PTH has no attention parameters for layer {layer}")
        stale += found
    if dry_run:
        return
    if not overwrite and any(p.exists() for p in (out, sidecar(out, "config"), sidecar(out, "manifest"))):
        raise FileExistsError("Output exists; choose a new --out or pass --overwrite")
    out.parent.mkdir(parents=True, exist_ok=True)
    if shutil.disk_usage(out.parent).free < base.stat().st_size + (512 << 20):
        raise OSError("Insufficient free disk space for a second PTH")
    rel_root = weights if weights.is_dir() else weights.parent
    by_file = defaultdict(list)
    for (layer, name), path in pick.items():
        by_file[path].append((layer, name))
    fresh, entries = {}, []
    for path in files:
        if path not in by_file:
            continue
        with safe_open(str(path), framework="pt", device="cpu") as f:
            for layer, name in sorted(by_file[path]):
                value = f.get_tensor(f"{layer}.{name}")
                if tuple(value.shape) != schemas[layer][name]:
                    raise ValueError(f"Tensor changed during conversion: {path}:{layer}.{name}")
                if dtype == "base":
                    value = value.to(base_dtype)
                value = export_tensor(name, value)
                target = f"blocks.{layer}.att.{name}"
                fresh[target] = value
                entries.append({"source": f"{layer}.{name}", "file": str(path.relative_to(rel_root)),
                                "target": target, "shape": list(value.shape),
                                "dtype": str(value.dtype).removeprefix("torch."),
                                "transform": ("transpose_out_in" if name in LOW_RANK else
                                              "squeeze_vector" if len(schemas[layer][name]) == 3 else "copy"),
                                "dtype_policy": dtype})
    for key in stale:
        del state[key]
    state.update(fresh)
    config.update(format=FORMAT, weights_file=out.name, exported_utc=datetime.now(timezone.utc).isoformat(),
                  requires_hybrid_backend=True)
    config.pop("requires_hybrid_timemix_dispatch", None)
    mixers = config.setdefault("timemix_layers", {})
    for layer in layers:
        kinds[layer] = TIMEMIX_KIND
        mixers[str(layer)] = {"head_size": sizes[layer], "num_heads": width // sizes[layer],
                              "source": "RWKV-Theseus TimeMix"}
    summary = config.setdefault("summary", {})
    summary.update(output_tensors=len(state), layer_counts=dict(Counter(kinds)), output=str(out))
    terms = config.setdefault("contract", {})
    terms.update({
        "checkpoint_linear_layout": "out_in_row_major", "timemix_weight_layout": "out_in_row_major_vectors_flat_v1",
        "timemix": ("RWKV-Theseus TimeMix; independent shift and FP32 WKV state per layer; GDN and TimeMix use "
                    "the same shared WKV kernel with per-layer D64/D128"),
        "wkv_kernel": "shared_dplr_fp32_v1", "wkv_state_layout": "B,H,K,V",
        "wkv_decay_input": "effective_multiplier",
        "wkv_decay_operation": "identity; decay is computed by the mixer adapter",
        "wkv_inputs": "r,decay,k,v,a,b: FP32 [B,T,H,D]; output: FP16",
        "gdn_wkv_inputs": "r=q/sqrt(D), decay=exp(g), k=k, v=beta*v, a=k, b=-exp(g)*beta*k",
        "timemix_wkv_inputs": "decay=exp(-0.6065306597126334*sigmoid(raw_w)); remaining inputs from TimeMix"})
    wkv = {}
    for i, kind in enumerate(kinds):
        if kind == TIMEMIX_KIND:
            heads, size = state[f"blocks.{i}.att.r_k"].shape
        elif kind == "linear_attention":
            heads, size = int(geo["linear_num_value_heads"]), int(geo["linear_key_head_dim"])
            if size not in (64, 128) or int(geo["linear_value_head_dim"]) != size:
                raise ValueError("Shared WKV requires square D64/D128 GDN states")
        else:
            continue
        wkv[str(i)] = {"kind": kind, "head_size": int(size), "num_heads": int(heads)}
    config["wkv_layers"] = wkv
    manifest["format"] = FORMAT
    manifest["tensors"] = [e for e in manifest["tensors"]
                           if not any(e["target"].startswith(f"blocks.{i}.att.") for i in layers)] + entries
    manifest["replaced_attention_layers"] = sorted(int(k) for k in mixers)
    tmp = _save_pth(state, out, quiet, verify)
    try:
        config["weights_bytes"] = os.path.getsize(tmp)
        atomic_json(sidecar(out, "config"), config)
        atomic_json(sidecar(out, "manifest"), manifest)
        os.replace(tmp, out)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)
    print(f"Saved: {out}\nConfig: {sidecar(out, 'config')}\nManifest: {sidecar(out, 'manifest')}")
