"""NOVA Winograd F(6,3) -- FP16 3x3 stride-1 convolution forward for NVIDIA B200.

Drop-in for the Python surface of Jayluci4/nova-wino-amd (``nova_winograd/__init__.py``):

    from nova_winograd import NovaWinogradConv2d, replace_conv2d_with_nova

    conv = NovaWinogradConv2d(64, 128, kernel_size=3, padding=1).cuda()
    y = conv(x_fp16)

    model = torchvision.models.resnet50().cuda().half()
    replace_conv2d_with_nova(model)

The arithmetic runs in ``lib/libnova_winograd.so`` (hand-written sm_100a CUDA:
transform kernels and a tcgen05/TMEM batched GEMM fed by TMA).
"""

from nova_winograd.conv2d import (
    NovaWinogradConv2d,
    NovaWinogradConv2dCompilable,
    NovaWinogradConv2dTrainable,
)
from nova_winograd.ops import compute_tiling, nova_forward
from nova_winograd.surgery import replace_conv2d_with_nova

__version__ = "0.1.0"
__all__ = [
    "NovaWinogradConv2d",
    "NovaWinogradConv2dTrainable",
    "NovaWinogradConv2dCompilable",
    "nova_forward",
    "compute_tiling",
    "replace_conv2d_with_nova",
]
