"""EXL3 layer packing, safetensors export and reload on B200.

Same names, arguments, tensor keys, shapes, dtypes and errors as the
reference ``exl3_quant/serialization.py``. The per-tile work (container
packing, unpacking, weight decode) runs in libexl3k kernels on the GPU:

* ``pack_module_trellis`` -> ``exl3_pack_trellis`` (pack_trellis + SWAP16 of
  every tile in one launch; serialization.py:40-62 loops over tiles in NumPy);
* ``unpack_module_trellis`` -> ``exl3_unpack_trellis`` (serialization.py:65-84);
* ``decode_weight_from_storage`` -> ``exl3_decode_weight``: states, codebook,
  inverse tile permutation and the two 128-block rotations with the scales
  in one pass (serialization.py:227-266).

The file format side (safetensors dictionaries, quantization_config.json,
the index file) is host code, as in the reference; tensors leave the GPU
once, already packed.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Dict, Optional, Tuple, Union

import torch

from ._ext import ext, require_cuda
from .trellis_format import CB_3INST, CB_MCG, CB_MUL1


def _on_cuda(t: torch.Tensor) -> torch.Tensor:
    dev = t.device if t.is_cuda else require_cuda(None)
    return t.to(dev)


def pack_module_trellis(encoded: torch.Tensor, K: int) -> torch.Tensor:
    """(tiles_k, tiles_n, 256) states -> (tiles_k, tiles_n, 16*K) int16
    container (serialization.py:40-62). The result stays on the GPU that
    packed it (the input's device, or the current CUDA device for a CPU
    input)."""
    if encoded.dim() != 3 or encoded.shape[-1] != 256:
        raise ValueError(
            f"encoded states must have shape (tiles_k, tiles_n, 256), got {tuple(encoded.shape)}")
    if not 1 <= int(K) <= 8:
        raise ValueError(f"K must be in 1..8, got {K}")
    tk, tn, _ = encoded.shape
    st = _on_cuda(encoded).to(torch.int16).contiguous()
    out = torch.empty((tk, tn, 16 * K), dtype=torch.int16, device=st.device)
    if st.numel():
        ext().pack_trellis(st.view(-1, 256), out.view(-1, 16 * K), int(K))
    return out


def unpack_module_trellis(trellis: torch.Tensor, K: int) -> torch.Tensor:
    """(tiles_k, tiles_n, 16*K) int16 container -> (tiles_k, tiles_n, 256)
    int16 states (serialization.py:65-84)."""
    if trellis.dim() != 3:
        raise ValueError(f"trellis must be 3-D, got {tuple(trellis.shape)}")
    tk, tn, pd = trellis.shape
    if pd != 16 * K:
        raise ValueError(f"Trellis last dimension {pd} does not match 16 * K = {16 * K}")
    tw = _on_cuda(trellis).to(torch.int16).contiguous()
    out = torch.empty((tk, tn, 256), dtype=torch.int16, device=tw.device)
    if tw.numel():
        ext().unpack_trellis(tw, out, int(K))
    return out


def decode_weight_from_storage(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
                               K: int, cb: int = CB_MUL1,
                               return_w_hat: bool = False):
    """Original-basis (k, n) fp32 weight from the stored trellis and scales
    (serialization.py:227-266): ``H_l(w_hat) * su -> H_r -> * sv``.

    ``suh``/``svh`` are the stored fp16 vectors (fp32 accepted). With
    ``return_w_hat`` the transformed-basis reconstruction is returned too.
    """
    if trellis.dim() != 3:
        raise ValueError(f"trellis must be 3-D, got {tuple(trellis.shape)}")
    tk, tn, pd = trellis.shape
    if pd != 16 * K:
        raise ValueError(f"Trellis last dimension {pd} does not match 16 * K = {16 * K}")
    k, n = tk * 16, tn * 16
    if suh.numel() != k or svh.numel() != n:
        raise ValueError(f"su must have {k} elements and sv {n}, got {suh.numel()} / {svh.numel()}")
    if k % 128 or n % 128:
        raise ValueError(f"weight dims ({k} x {n}) must be multiples of 128")
    if cb not in (CB_3INST, CB_MCG, CB_MUL1):
        raise ValueError(f"Unknown codebook {cb}")
    tw = _on_cuda(trellis).to(torch.int16).contiguous()
    dev = tw.device
    sdt = torch.float32 if (suh.dtype == torch.float32 and svh.dtype == torch.float32) \
        else torch.float16
    su = suh.reshape(-1).to(device=dev, dtype=sdt).contiguous()
    sv = svh.reshape(-1).to(device=dev, dtype=sdt).contiguous()
    out = torch.empty((k, n), dtype=torch.float32, device=dev)
    w_hat = torch.empty((k, n), dtype=torch.float32, device=dev) if return_w_hat else None
    ext().decode_weight(tw, su, sv, out, w_hat, int(K), int(cb))
    return (out, w_hat) if return_w_hat else out


def _codebook_name(cb: int) -> str:
    return "mul1" if cb == CB_MUL1 else ("mcg" if cb == CB_MCG else "3inst")


def build_layer_tensors(module_results: Dict[str, Any], layer_idx: int = 0,
                        prefix: str = "model.layers",
                        norm_weights: Optional[Dict[str, torch.Tensor]] = None,
                        extra_tensors: Optional[Dict[str, torch.Tensor]] = None,
                        preserve_source_dtype: bool = False
                        ) -> Tuple[Dict[str, torch.Tensor], Dict[str, Any]]:
    """EXL3 safetensors dictionary and per-module metadata for one layer
    (serialization.py:87-170): ``<prefix>.<layer>.<module>.trellis`` (int16
    (tiles_k, tiles_n, 16K)), ``.suh`` (fp16 (k,)), ``.svh`` (fp16 (n,)) and
    the codebook marker (``.mul1`` / ``.mcg`` int32 scalar; none for 3INST).
    Packing and the fp16 casts run on the GPU; each tensor is copied to the
    host once."""
    tensors: Dict[str, torch.Tensor] = {}
    storage: Dict[str, Any] = {}
    layer_prefix = f"{prefix}.{layer_idx}" if prefix else f"layers.{layer_idx}"
    for name, res in module_results.items():
        mod_key = f"{layer_prefix}.{name}"
        trellis = pack_module_trellis(res.encoded, K=res.K)
        suh = res.su.detach().flatten().to(torch.float16)
        svh = res.sv.detach().flatten().to(torch.float16)
        tensors[f"{mod_key}.trellis"] = trellis.cpu()
        tensors[f"{mod_key}.suh"] = suh.cpu()
        tensors[f"{mod_key}.svh"] = svh.cpu()
        if res.cb == CB_MUL1:
            tensors[f"{mod_key}.mul1"] = torch.tensor(0, dtype=torch.int32)
        elif res.cb == CB_MCG:
            tensors[f"{mod_key}.mcg"] = torch.tensor(0, dtype=torch.int32)
        storage[mod_key] = {
            "quant_format": "exl3",
            "bits_per_weight": res.K,
            "codebook": _codebook_name(res.cb),
            "stored_tensors": {
                f"{mod_key}.trellis": {"shape": list(trellis.shape)},
                f"{mod_key}.suh": {"shape": list(suh.shape)},
                f"{mod_key}.svh": {"shape": list(svh.shape)},
            },
        }
    if norm_weights:
        for norm_name, w in norm_weights.items():
            cw = w.detach().cpu()
            tensors[f"{layer_prefix}.{norm_name}"] = cw if preserve_source_dtype \
                else cw.to(torch.float16)
    if extra_tensors:
        for key, w in extra_tensors.items():
            if key in tensors:
                raise ValueError(f"pass-through tensor collides with an emitted tensor: {key}")
            tensors[key] = w.detach().cpu()
    return tensors, storage


def export_layer_safetensors(module_results: Dict[str, Any], output_dir: Union[str, Path],
                             filename: str = "model.safetensors", layer_idx: int = 0,
                             prefix: str = "model.layers",
                             norm_weights: Optional[Dict[str, torch.Tensor]] = None
                             ) -> Tuple[Path, Path]:
    """Write the layer's tensors, ``quantization_config.json`` and the
    ``model.safetensors.index.json`` weight map (serialization.py:173-224)."""
    from safetensors.torch import save_file

    out_dir = Path(output_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    tensors, storage = build_layer_tensors(module_results, layer_idx=layer_idx, prefix=prefix,
                                           norm_weights=norm_weights)
    sample = next(iter(module_results.values()))
    meta = {
        "quant_format": "exl3",
        "producer": "EXL3_Intel_Arc_quantizer",
        "version": "1.0",
        "codebook": "mul1" if sample.cb == CB_MUL1 else "3inst",
        "bits": str(sample.K),
    }
    st_file = out_dir / filename
    save_file(tensors, str(st_file), metadata=meta)
    qc_file = out_dir / "quantization_config.json"
    qc_file.write_text(json.dumps({"quant_method": "exl3", "bits": sample.K,
                                   "codebook": meta["codebook"], "tensor_storage": storage},
                                  indent=2))
    (out_dir / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": meta, "weight_map": {k: filename for k in tensors}}, indent=2))
    return st_file, qc_file


def load_and_verify_layer_safetensors(safetensors_path: Union[str, Path],
                                      expected_results: Optional[Dict[str, Any]] = None,
                                      atol: float = 5e-3) -> Dict[str, torch.Tensor]:
    """Reload a layer file and decode every module on the GPU
    (serialization.py:269-320); with ``expected_results`` each decoded
    weight must match the module's ``w_hat`` within ``atol``."""
    from safetensors import safe_open

    path = Path(safetensors_path)
    if not path.exists():
        raise FileNotFoundError(f"Safetensors file not found: {path}")
    with safe_open(str(path), framework="pt", device="cpu") as f:
        loaded = {k: f.get_tensor(k) for k in f.keys()}
    out: Dict[str, torch.Tensor] = {}
    for t_key in [k for k in loaded if k.endswith(".trellis")]:
        mod = t_key[:-len(".trellis")]
        if f"{mod}.suh" not in loaded or f"{mod}.svh" not in loaded:
            raise KeyError(f"Missing suh or svh for {mod}")
        trellis = loaded[t_key]
        K = trellis.shape[-1] // 16
        cb = CB_MCG if f"{mod}.mcg" in loaded else (CB_MUL1 if f"{mod}.mul1" in loaded else CB_3INST)
        w = decode_weight_from_storage(trellis, loaded[f"{mod}.suh"], loaded[f"{mod}.svh"],
                                       K=K, cb=cb)
        out[mod] = w
        if expected_results:
            for name, res in expected_results.items():
                if name in mod:
                    diff = float((w - res.w_hat.to(w.device).float()).abs().max())
                    assert diff < atol, \
                        f"Mismatch in reloaded {name}: max diff {diff} exceeds atol {atol}"
    return out
