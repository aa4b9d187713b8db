"""Quantised checkpoints: save a swapped model's int4 weights, load them into a fresh one.

The reference keeps only the in-memory swap (src/w4a16/kernels.py:127-137): every load of
a model re-reads the dense fp16 weights and re-runs the CPU quantiser and packer
(kernels.py:47-91).  Here a model whose Linears are W4A16Linear can be saved as its packed
codes, scales and biases (0.5 B per weight plus scales, no dense copy), and a model built
with the same architecture (any initialisation) gets them back without quantising again.

File format (torch.save of a dict):
    {"format": "w4a16-b200/1",
     "linears": {qualified name: {"packed": uint8 [out, in/2] (interleaved packing),
                                   "scale": fp32/fp16 [out] or [out, in/128],
                                   "bias": tensor or None}},
     "state": every other entry of the model's state_dict}
"""
import torch
import torch.nn as nn

from .linear import W4A16Linear

FORMAT = "w4a16-b200/1"


def _named_w4a16(module):
    return [(name, m) for name, m in module.named_modules() if isinstance(m, W4A16Linear)]


def save_quantized(module, path):
    """Write the W4A16Linear weights of `module` and the rest of its state to `path`."""
    lin = _named_w4a16(module)
    if not lin:
        raise ValueError("the module has no W4A16Linear layers (swap them in first)")
    linears = {}
    skip = set()
    for name, m in lin:
        linears[name] = {"packed": m.packed.detach().cpu(), "scale": m.scale.detach().cpu(),
                         "bias": None if m.bias is None else m.bias.detach().cpu()}
        prefix = name + "." if name else ""
        skip.update(prefix + k for k in ("packed", "scale", "dense_weight", "bias"))
    state = {k: v.detach().cpu() for k, v in module.state_dict().items() if k not in skip}
    torch.save({"format": FORMAT, "linears": linears, "state": state}, path)


def _set_child(root, qualified, child):
    parent = root
    parts = qualified.split(".")
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], child)


def load_quantized(module, path, device=None):
    """Replace the Linears named in the checkpoint with W4A16Linear built from the stored
    codes (no dense weight, no quantisation) and load the remaining state.

    `module` is the same architecture with any weights (e.g. a freshly constructed model);
    device places the buffers (default: the current CUDA device).  Every checkpoint
    entry must find its place and every non-swapped parameter must be in the checkpoint."""
    ck = torch.load(path, map_location="cpu", weights_only=True)
    if ck.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    modules = dict(module.named_modules())
    for name, ent in ck["linears"].items():
        if not name:
            raise KeyError("the root module itself cannot be swapped in place")
        old = modules.get(name)
        if not isinstance(old, (nn.Linear, W4A16Linear)):
            raise KeyError(f"checkpoint layer {name!r} is not a Linear in this model")
        packed, scale = ent["packed"], ent["scale"]
        if (packed.shape[0], packed.shape[1] * 2) != (old.out_features, old.in_features):
            raise ValueError(f"{name}: checkpoint shape {tuple(packed.shape)} does not match "
                             f"{old.out_features} x {old.in_features}")
        bias = None
        if ent["bias"] is not None:
            bias = nn.Parameter(ent["bias"].to(dev), requires_grad=False)
        _set_child(module, name, W4A16Linear(None, bias, packed.to(dev), scale.to(dev)))
    missing, unexpected = module.load_state_dict(ck["state"], strict=False)
    swapped = set(ck["linears"])
    missing = [k for k in missing if k.rsplit(".", 1)[0] not in swapped]
    if missing or unexpected:
        raise KeyError(f"state mismatch: missing {missing[:5]}, unexpected {unexpected[:5]}")
    return module
