"""Checkpoint / resume of Concord-packed models, and export to plain layers.

The reference keeps two kinds of saves (its CLAUDE.md, "checkpoint duality";
concord/packed_b.py:1605-1649): backups carry the full packed state -- the
registered buffers of every packed layer (packed_w, row/col exponents, the
v-hat state, the rebalance high-watermarks and seed, lr/eps) -- and resume
re-materializes the bf16 forward weight from packed_w; final saves
consolidate every packed layer back into a standard nn.Linear / nn.Conv2d
(s_fast dropped: consolidated_weight()).

Some optimizer state is not in state_dict(), in the reference as here: the
per-device step salt (the SR-hash salt every apply launch on a device bumps
once, packed_b.py:315-322, 910-911), each layer's coh_pre gate EMA (a plain
attribute, packed_b.py:1467), the bf16 forward weight as the last step
emitted it, the layer knobs a trainer or the autotuner
changes during a run (gf_consol, beta1, lr, ...) and the module-wide gate
settings (set_fixed_coh, set_gate_gain, set_ratio_coh(_floors)).  A resumed
run reproduces the uninterrupted run's words bit for bit only when all of
them are restored, so `save_state` / `load_state` carry them.

For a row-sharded data-parallel layer call RowShardedStep.gather_state()
first: it makes the packed state of every rank complete.
"""
import copy

import torch

from . import packed_b as _pb

FORMAT = "concord_b200/checkpoint/1"


def packed_layers(model):
    """(name, module) of every Concord-packed layer of `model`."""
    for name, m in model.named_modules():
        if isinstance(m, (_pb.ConcordLinearPackedB, _pb.ConcordConv2dPackedB)):
            yield name, m


def _devices(model):
    return sorted({_pb._dev_key(m.packed_w.device) for _, m in packed_layers(model)})


def get_step_salt(device):
    """The per-device step salt (an int; reads the device)."""
    return int(_pb._get_step_counter(torch.device(device)).item())


def set_step_salt(device, value):
    """Set the per-device step salt (stream-ordered fill)."""
    _pb._get_step_counter(torch.device(device)).fill_(int(value))


# layer attributes that steer the step and are not buffers
_KNOBS = ("alpha", "beta1", "optimizer_kind", "weight_decay", "_eps_value", "_lr_value", "step_cap",
          "v_scale", "precond_p", "gf_consol", "fast_gain", "alpha_v_fast", "drift_cancel_C",
          "track_adafactor_v", "adafactor_beta2", "gf_trust_delta_sq", "allow_tickdown", "wd_sv",
          "wd_sf", "mass_preserve_v", "apply_chase", "track_rebalance")
_GLOBALS = ("_USE_FIXED_COH", "_GATE_GAIN", "_COH_WEIGHTED_V", "_RATIO_COH", "_RATIO_CHASE_FLOOR",
            "_RATIO_LEAK_FLOOR", "_FLOOR_TENSORS_ON", "_SIGMAG_NOISE", "_SIGMAG_ISO", "_SIGMAG_SIGMA", "_CONV_BACKEND")


def save_state(model):
    """Everything needed to resume bit-exactly: the module's state_dict (packed
    buffers included), each packed layer's coh_pre and knobs, the module-wide
    gate settings and the step salt of every device a packed layer lives on."""
    layers = {}
    for name, m in packed_layers(model):
        cp = m._coh_pre
        wb = getattr(m, "_bf16_weight_buf", None)
        layers[name] = {"coh_pre": None if cp is None else cp.detach().clone(),
                        "weight_buf": None if wb is None else wb.detach().clone(),
                        "knobs": {k: getattr(m, k) for k in _KNOBS if hasattr(m, k)}}
    return {"format": FORMAT,
            "model": model.state_dict(),
            "layers": layers,
            "globals": {k: getattr(_pb, k) for k in _GLOBALS},
            "step_salt": {dev: get_step_salt(dev) for dev in _devices(model)}}


@torch.no_grad()
def load_state(model, state, strict=True):
    """Restore `save_state` output into a model of the same architecture:
    buffers, coh_pre, knobs, gate settings, step salts and every layer's bf16
    forward weight.  The forward weight is the saved one: the step emits it
    and the rebalance that follows does not refresh it, so re-deriving it
    from the words (the reference's resync, used when it was not saved) can
    differ from what the uninterrupted run reads next."""
    if state.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    missing, unexpected = model.load_state_dict(state["model"], strict=strict)
    saved = state.get("layers", {})
    for name, m in packed_layers(model):
        extra = saved.get(name)
        if extra is not None:
            for k, v in extra["knobs"].items():
                setattr(m, k, v)
            m.lr, m.eps = m._lr_value, m._eps_value        # refill the device scalars
            cp = extra["coh_pre"]
            if cp is None:
                m.disable_cohpre()
            else:
                m.enable_cohpre().copy_(cp)
        wb = None if extra is None else extra.get("weight_buf")
        if wb is not None:
            m._ensure_buffers()[0].copy_(wb)
        else:
            m._resync_weight_buf()
    for k, v in state.get("globals", {}).items():
        setattr(_pb, k, v)
    for dev, salt in state.get("step_salt", {}).items():
        set_step_salt(dev, salt)
    return missing, unexpected


@torch.no_grad()
def export_dense(model, dtype=torch.bfloat16):
    """A copy of `model` with every packed layer replaced by the plain layer it
    deploys as: nn.Linear / nn.Conv2d holding consolidated_weight() (the slow
    accumulators, s_fast dropped) in `dtype`, bias copied.  The original model
    is untouched."""
    out = copy.deepcopy(model)
    for name, m in list(packed_layers(out)):
        dev = m.packed_w.device
        w = m.consolidated_weight().to(dtype)
        bias = getattr(m, "bias", None)
        if isinstance(m, _pb.ConcordConv2dPackedB):   # (a subclass of the linear layer)
            dense = torch.nn.Conv2d(m.in_channels, m.out_channels, (m.kh, m.kw), stride=m.stride,
                                    padding=m.padding, bias=bias is not None, device=dev,
                                    dtype=dtype)
            dense.weight.copy_(w.view(m.out_channels, m.in_channels, m.kh, m.kw))
        else:
            dense = torch.nn.Linear(m.in_features, m.out_features, bias=bias is not None,
                                    device=dev, dtype=dtype)
            dense.weight.copy_(w)
        if bias is not None:
            dense.bias.copy_(bias.detach().to(dtype))
        if not name:            # the model is itself one packed layer
            return dense
        parent, _, leaf = name.rpartition(".")
        setattr(out.get_submodule(parent) if parent else out, leaf, dense)
    return out


@torch.no_grad()
def dense_state_dict(model, dtype=torch.bfloat16):
    """The state_dict of export_dense(model) without copying the model: every
    packed layer contributes `<name>.weight` (its consolidated_weight(), 4-D for
    convolutions) and `<name>.bias`, in `dtype`; every other parameter and
    buffer is taken as it is."""
    packed = dict(packed_layers(model))
    out = {}
    for name, m in packed.items():
        pre = name + "." if name else ""
        w = m.consolidated_weight().to(dtype)
        if isinstance(m, _pb.ConcordConv2dPackedB):
            w = w.view(m.out_channels, m.in_channels, m.kh, m.kw)
        out[pre + "weight"] = w
        if getattr(m, "bias", None) is not None:
            out[pre + "bias"] = m.bias.detach().to(dtype)
    for k, v in model.state_dict().items():
        if k.rpartition(".")[0] in packed:      # a packed layer's own buffers
            continue
        out[k] = v.detach()
    return out


def save_consolidated(model, path, dtype=torch.bfloat16):
    """Write the deployable dense weights as a safetensors file (the
    reference's final save: packed layers consolidated back to plain
    Linear / Conv2d weights, so the checkpoint loads as the ordinary model)."""
    from safetensors.torch import save_file
    sd = {k: v.contiguous().cpu() for k, v in dense_state_dict(model, dtype).items()}
    save_file(sd, path)
    return sorted(sd)
