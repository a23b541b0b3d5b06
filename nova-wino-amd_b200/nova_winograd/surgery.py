"""Model surgery: swap eligible ``nn.Conv2d`` layers for NOVA Winograd layers.

Same contract as the reference (Jayluci4/nova-wino-amd ``nova_winograd/surgery.py:9-53``):
a layer is eligible when kernel_size == (3, 3), stride == (1, 1),
dilation == (1, 1) and groups == 1; replacement happens in place and the
number of replaced layers is returned.
"""

import torch.nn as nn

from nova_winograd.conv2d import NovaWinogradConv2d, NovaWinogradConv2dTrainable


def is_eligible(module):
    """True for a Conv2d the NOVA F(6,3) kernel computes exactly (surgery.py:38)."""
    return (isinstance(module, nn.Conv2d)
            and not isinstance(module, NovaWinogradConv2d)
            and module.kernel_size == (3, 3) and module.stride == (1, 1)
            and module.dilation == (1, 1) and module.groups == 1
            and not isinstance(module.padding, str)
            and module.padding[0] == module.padding[1]
            and module.padding_mode == "zeros")


def replace_conv2d_with_nova(model, trainable=False, verbose=True):
    """Replace every eligible nn.Conv2d of ``model`` in place.

    Args:
        model:     nn.Module to modify.
        trainable: use NovaWinogradConv2dTrainable (supports backward).
        verbose:   print a one-line summary.

    Returns:
        Number of layers replaced.
    """
    cls = NovaWinogradConv2dTrainable if trainable else NovaWinogradConv2d
    replaced = skipped = 0
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Conv2d) or isinstance(module, NovaWinogradConv2d):
            continue
        if not is_eligible(module):
            skipped += 1
            continue
        parent_name, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, attr, cls.from_conv2d(module))
        replaced += 1
    if verbose:
        print(f"NOVA: replaced {replaced} Conv2d layers, skipped {skipped} ineligible")
    return replaced
