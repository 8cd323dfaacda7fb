"""Put Concord on an existing model: swap its nn.Linear (and, optionally,
nn.Conv2d) modules for ConcordLinearPackedB / ConcordConv2dPackedB, each
loaded with the module's current weight, the way the reference's trainers do
it (notebook/src/train_nanogpt.py:140-170, notebook/src/sdxl_train.py:103-127).
Everything else (embeddings, norms, biases) stays an ordinary parameter for
an auxiliary optimizer.
"""
import torch
import torch.nn as nn

from .packed_b import ConcordConv2dPackedB, ConcordLinearPackedB


@torch.no_grad()
def concordify(model, lr, convs=False, finetune=False, skip=None, device=None):
    """Replace every nn.Linear (and nn.Conv2d with groups == 1 when `convs`)
    in `model` by the packed layer, in place; returns the list of new layers.

    `finetune` loads with load_weights_finetune (pretrained weights at the
    steady state) instead of load_weights (the whole weight in the fast
    accumulator, the from-scratch recipe).  `skip(name, module)` may return
    True to leave a module alone."""
    made = []
    for parent_name, parent in list(model.named_modules()):
        for name, child in list(parent.named_children()):
            full = f"{parent_name}.{name}" if parent_name else name
            if skip is not None and skip(full, child):
                continue
            dev = device or (child.weight.device if hasattr(child, "weight") else None)
            if isinstance(child, nn.Linear):
                new = ConcordLinearPackedB(child.in_features, child.out_features,
                                           bias=child.bias is not None, device=dev, lr=lr)
                W = child.weight.float()
            elif convs and isinstance(child, nn.Conv2d) and child.groups == 1 and \
                    child.dilation == (1, 1) and child.padding_mode == "zeros" and \
                    child.stride[0] == child.stride[1] and child.padding[0] == child.padding[1] and \
                    child.kernel_size[0] == child.kernel_size[1]:
                new = ConcordConv2dPackedB(child.in_channels, child.out_channels, child.kernel_size[0],
                                           stride=child.stride[0], padding=child.padding[0],
                                           bias=child.bias is not None, device=dev, lr=lr)
                W = child.weight.float().reshape(child.out_channels, -1)
            else:
                continue
            (new.load_weights_finetune if finetune else new.load_weights)(W)
            if child.bias is not None:
                new.bias.copy_(child.bias.float())
            setattr(parent, name, new)
            made.append(new)
    return made


def concord_layers(model):
    return [m for m in model.modules() if isinstance(m, (ConcordLinearPackedB, ConcordConv2dPackedB))]


def aux_parameters(model):
    """The parameters Concord does not step (embeddings, norms, biases)."""
    return [p for p in model.parameters() if p.requires_grad]
