"""Tensor inventory of the PP-OCRv6 detector and recognizer checkpoints.

The names and shapes are the ones the reference loaders look up
(ppocr-rs src/cpu/model.rs:1546-1609 for the detector, 1961-2022 for the
recognizer, with the block tables at 1648-1680 and 2042-2122).  Every entry
carries a ``role`` that the seeded generator uses to pick a distribution:

    conv     convolution or linear kernel (fan-in scaled)
    bias     additive bias of a conv / linear
    bn.*     batch-norm gamma / beta / running_mean / running_var
    ln.*     layer-norm weight / bias
    rank1    dense 9x9 kernel that must factor as p[o,i] * d[i,:,:]

Tensor counts per tier match the reference's load-time check
(src/gpu/model.rs:11-16): detectors 350/271/271, recognizers 269/250/150.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

DETECTOR_TENSORS = {"medium": 350, "small": 271, "tiny": 271}
RECOGNIZER_TENSORS = {"medium": 269, "small": 250, "tiny": 150}
RECOGNIZER_CLASSES = {"medium": 18710, "small": 18710, "tiny": 6906}

# Stage channel tables (src/cpu/model.rs:1553-1601).
DETECTOR_STAGE_CHANNELS = {
    "medium": (128, 256, 512, 896),
    "small": (48, 96, 192, 384),
    "tiny": (32, 48, 64, 160),
}
DETECTOR_STEM = {"medium": (64, 128), "small": (24, 48), "tiny": (16, 32)}
# RepLkFpn (neck channels, depthwise kernel) for small/tiny (src/cpu/model.rs:1578-1599).
DETECTOR_FPN = {"small": (96, 7), "tiny": (64, 5)}
DETECTOR_NECK_CHANNELS = {"medium": 256, "small": 96, "tiny": 64}


@dataclass(frozen=True)
class Block:
    kernel: int
    cin: int
    cout: int
    stride: Tuple[int, int]
    se: bool

    @property
    def residual(self) -> bool:
        # src/cpu/model.rs:528
        return self.cin == self.cout and self.stride == (1, 1)


def _b(cin: int, cout: int, stride: Tuple[int, int], se: bool) -> Block:
    return Block(3, cin, cout, stride, se)


def detector_stages(size: str) -> List[List[Block]]:
    """Four LCNet stages of the detector backbone (src/cpu/model.rs:1648-1680)."""
    s1, s2, s3, s4 = DETECTOR_STAGE_CHANNELS[size]
    return [
        [_b(s1, s1, (1, 1), True), _b(s1, s1, (1, 1), False)],
        [_b(s1, s2, (2, 2), False), _b(s2, s2, (1, 1), True), _b(s2, s2, (1, 1), False)],
        [
            _b(s2, s3, (2, 2), False),
            _b(s3, s3, (1, 1), True),
            _b(s3, s3, (1, 1), False),
            _b(s3, s3, (1, 1), True),
            _b(s3, s3, (1, 1), False),
        ],
        [_b(s3, s4, (2, 2), False), _b(s4, s4, (1, 1), True), _b(s4, s4, (1, 1), False)],
    ]


def recognizer_stages(size: str) -> List[List[Block]]:
    """LCNet stages of the recognizer backbones (src/cpu/model.rs:2057-2122)."""
    if size == "medium":
        return [
            [_b(128, 128, (1, 1), True)],
            [_b(128, 256, (1, 1), False), _b(256, 256, (1, 1), False), _b(256, 256, (1, 1), True)],
            [_b(256, 512, (2, 1), False)]
            + [_b(512, 512, (1, 1), i % 2 == 0) for i in range(6)],
            [_b(512, 768, (2, 1), False), _b(768, 768, (1, 1), True), _b(768, 768, (1, 1), False)],
        ]
    if size == "small":
        return [
            [_b(96, 96, (1, 1), True)],
            [_b(96, 96, (1, 1), False), _b(96, 96, (1, 1), False)],
            [_b(96, 192, (2, 1), False)]
            + [_b(192, 192, (1, 1), i % 2 == 0) for i in range(6)],
            [_b(192, 384, (2, 1), False), _b(384, 384, (1, 1), True), _b(384, 384, (1, 1), False)],
        ]
    if size == "tiny":
        return [
            [_b(48, 48, (1, 1), True)],
            [_b(48, 48, (1, 1), False)],
            [_b(48, 96, (2, 1), False), _b(96, 96, (1, 1), True), _b(96, 96, (1, 1), False)],
            [
                _b(96, 160, (2, 1), False),
                _b(160, 160, (1, 1), True),
                _b(160, 160, (1, 1), False),
                _b(160, 160, (1, 1), False),
            ],
        ]
    raise ValueError(f"unknown model size {size!r}")


# Recognizer stem kind and widths (src/cpu/model.rs:1968-2018).
RECOGNIZER_STEM = {"medium": ("large", 64, 128), "small": ("large", 48, 96), "tiny": ("small", 24, 48)}
# LightSVTR head: (input channels, hidden, mlp) for medium/small (src/cpu/model.rs:1977-1998).
RECOGNIZER_SVTR = {"medium": (768, 192, 768), "small": (384, 120, 240)}
RECOGNIZER_HEADS = 8
RECOGNIZER_DEPTH = 2


class _Inventory:
    def __init__(self) -> None:
        self.items: Dict[str, Tuple[Tuple[int, ...], str, int]] = {}

    def add(self, name: str, shape, role: str, fan_in: int = 0) -> None:
        if name in self.items:
            raise ValueError(f"duplicate tensor {name}")
        self.items[name] = (tuple(int(v) for v in shape), role, int(fan_in))

    def conv(self, prefix: str, cout: int, cin_per_group: int, kh: int, kw: int, bias: bool) -> None:
        self.add(f"{prefix}.weight", (cout, cin_per_group, kh, kw), "conv", cin_per_group * kh * kw)
        if bias:
            self.add(f"{prefix}.bias", (cout,), "bias")

    def bn(self, prefix: str, channels: int) -> None:
        self.add(f"{prefix}.weight", (channels,), "bn.gamma")
        self.add(f"{prefix}.bias", (channels,), "bn.beta")
        self.add(f"{prefix}.running_mean", (channels,), "bn.mean")
        self.add(f"{prefix}.running_var", (channels,), "bn.var")

    def conv_bn(self, prefix: str, cout: int, cin_per_group: int, kh: int, kw: int, norm: str = "normalization", bias: bool = False) -> None:
        self.conv(f"{prefix}.convolution", cout, cin_per_group, kh, kw, bias)
        self.bn(f"{prefix}.{norm}", cout)

    def linear(self, prefix: str, cin: int, cout: int) -> None:
        self.add(f"{prefix}.weight", (cout, cin), "conv", cin)
        self.add(f"{prefix}.bias", (cout,), "bias")

    def layer_norm(self, prefix: str, features: int) -> None:
        self.add(f"{prefix}.weight", (features,), "ln.weight")
        self.add(f"{prefix}.bias", (features,), "ln.bias")


def _lcnet_block(inv: _Inventory, prefix: str, block: Block) -> None:
    # src/cpu/model.rs:526-587
    if block.residual:
        inv.conv(f"{prefix}.token_conv", block.cout, 1, block.kernel, block.kernel, True)
    else:
        inv.conv_bn(f"{prefix}.token_conv", block.cin, 1, block.kernel, block.kernel)
    if block.se:
        c = block.cin
        inv.conv(f"{prefix}.token_squeeze_excitation.convolutions.0", c // 4, c, 1, 1, True)
        inv.conv(f"{prefix}.token_squeeze_excitation.convolutions.2", c, c // 4, 1, 1, True)
    inv.conv_bn(f"{prefix}.channel_conv1", block.cin * 2, block.cin, 1, 1)
    inv.conv_bn(f"{prefix}.channel_conv2", block.cout, block.cin * 2, 1, 1)


def _large_stem(inv: _Inventory, prefix: str, mid: int, out: int) -> None:
    # src/cpu/model.rs:626-683
    inv.conv_bn(f"{prefix}.stem1", mid, 3, 3, 3)
    inv.conv_bn(f"{prefix}.stem2a", mid // 2, mid, 2, 2)
    inv.conv_bn(f"{prefix}.stem2b", mid, mid // 2, 2, 2)
    inv.conv_bn(f"{prefix}.stem3", mid, mid * 2, 3, 3)
    inv.conv_bn(f"{prefix}.stem4", out, mid, 1, 1)


def _small_stem(inv: _Inventory, prefix: str, mid: int, out: int) -> None:
    # src/cpu/model.rs:695-728
    inv.conv_bn(f"{prefix}.conv1", mid, 3, 3, 3)
    inv.conv_bn(f"{prefix}.conv2", out, mid, 3, 3)


def _backbone(inv: _Inventory, stages: List[List[Block]], stem: Tuple[str, int, int]) -> None:
    enc = "model.backbone.encoder"
    kind, mid, out = stem
    if kind == "large":
        _large_stem(inv, f"{enc}.convolution", mid, out)
    else:
        _small_stem(inv, f"{enc}.convolution", mid, out)
    for si, stage in enumerate(stages):
        for bi, block in enumerate(stage):
            _lcnet_block(inv, f"{enc}.blocks.{si}.blocks.{bi}", block)


def _variant_se(inv: _Inventory, prefix: str, channels: int, reduction: int) -> None:
    # src/cpu/model.rs:1069-1096
    inv.conv(f"{prefix}.conv1", channels // reduction, channels, 1, 1, True)
    inv.conv(f"{prefix}.conv2", channels, channels // reduction, 1, 1, True)


def _rep_lk_fpn(inv: _Inventory, stage_channels, neck: int, kernel: int) -> None:
    # src/cpu/model.rs:1197-1232 (ResidualSqueezeExcitation 1107-1143, DepthwiseSeparableConv 1145-1195)
    for i, c in enumerate(stage_channels):
        inv.conv(f"model.neck.insert_conv.{i}.in_conv", neck, c, 1, 1, False)
        _variant_se(inv, f"model.neck.insert_conv.{i}.squeeze_excitation_block", neck, 4)
    for i in range(4):
        p = f"model.neck.input_conv.{i}"
        inv.conv(f"{p}.depthwise_convolution", neck, 1, kernel, kernel, True)
        inv.conv(f"{p}.pointwise_convolution", neck // 4, neck, 1, 1, False)
        _variant_se(inv, f"{p}.squeeze_excitation_module", neck // 4, 4)


def _medium_neck(inv: _Inventory) -> None:
    # src/cpu/model.rs:948-1020 and IntraclassBlock 890-937
    for i, c in enumerate((128, 256, 512, 896)):
        inv.conv(f"model.neck.input_channel_adjustment_convolution.{i}", 256, c, 1, 1, False)
    for i in range(4):
        inv.add(f"model.neck.input_feature_projection_convolution.{i}.weight", (64, 256, 9, 9), "rank1", 256 * 81)
        inv.add(f"model.neck.input_feature_projection_convolution.{i}.bias", (64,), "bias")
    for i in range(3):
        inv.conv(f"model.neck.path_aggregation_head_convolution.{i}", 64, 64, 3, 3, False)
    for i in range(4):
        inv.add(f"model.neck.path_aggregation_lateral_convolution.{i}.weight", (64, 64, 9, 9), "rank1", 64 * 81)
        inv.add(f"model.neck.path_aggregation_lateral_convolution.{i}.bias", (64,), "bias")
    for i in range(4):
        p = f"model.neck.intraclass_blocks.{i}"
        inv.conv(f"{p}.conv_reduce_channel", 32, 64, 1, 1, True)
        for ratio, k in (("longratio", 7), ("midratio", 5), ("shortratio", 3)):
            inv.conv(f"{p}.symmetric_conv_long_{ratio}", 32, 32, k, k, True)
            inv.conv(f"{p}.vertical_long_to_small_conv_{ratio}", 32, 32, k, 1, True)
            inv.conv(f"{p}.horizontal_small_to_long_conv_{ratio}", 32, 32, 1, k, True)
        inv.conv_bn(f"{p}.conv_final", 64, 32, 1, 1, norm="norm", bias=True)


def _detector_head(inv: _Inventory, channels: int) -> None:
    # src/cpu/model.rs:1479-1514
    hidden = channels // 4
    inv.conv_bn("head.conv_down", hidden, channels, 3, 3, norm="norm")
    inv.add("head.conv_up.convolution.weight", (hidden, hidden, 2, 2), "conv", hidden * 4)
    inv.add("head.conv_up.convolution.bias", (hidden,), "bias")
    inv.bn("head.conv_up.norm", hidden)
    inv.add("head.conv_final.weight", (hidden, 1, 2, 2), "conv", hidden * 4)
    inv.add("head.conv_final.bias", (1,), "bias")


def detector_inventory(size: str) -> Dict[str, Tuple[Tuple[int, ...], str, int]]:
    inv = _Inventory()
    mid, out = DETECTOR_STEM[size]
    _backbone(inv, detector_stages(size), ("large", mid, out))
    if size == "medium":
        _medium_neck(inv)
    else:
        neck, kernel = DETECTOR_FPN[size]
        _rep_lk_fpn(inv, DETECTOR_STAGE_CHANNELS[size], neck, kernel)
    _detector_head(inv, DETECTOR_NECK_CHANNELS[size])
    return inv.items


def recognizer_inventory(size: str) -> Dict[str, Tuple[Tuple[int, ...], str, int]]:
    inv = _Inventory()
    _backbone(inv, recognizer_stages(size), RECOGNIZER_STEM[size])
    classes = RECOGNIZER_CLASSES[size]
    if size == "tiny":
        # TinyRecognizerHead (src/cpu/model.rs:1913-1928); Conv1dBn weights are rank 3.
        inv.add("head.conv1.weight", (160, 1, 5), "conv", 5)
        inv.bn("head.norm1", 160)
        inv.add("head.conv2.weight", (160, 160, 1), "conv", 160)
        inv.bn("head.norm2", 160)
        inv.linear("head.fc1", 160, 80)
        inv.linear("head.fc2", 80, classes)
    else:
        cin, hidden, mlp = RECOGNIZER_SVTR[size]
        enc = "head.encoder"
        inv.conv_bn(f"{enc}.conv_block.0", hidden, cin, 1, 1)
        inv.conv_bn(f"{enc}.conv_block.1", hidden, cin, 1, 1)
        inv.conv_bn(f"{enc}.conv_block.2", hidden, 1, 1, 7)
        for i in range(RECOGNIZER_DEPTH):
            p = f"{enc}.svtr_block.{i}"
            inv.layer_norm(f"{p}.layer_norm1", hidden)
            inv.linear(f"{p}.self_attn.qkv", hidden, hidden * 3)
            inv.linear(f"{p}.self_attn.projection", hidden, hidden)
            inv.layer_norm(f"{p}.layer_norm2", hidden)
            inv.linear(f"{p}.mlp.fc1", hidden, mlp)
            inv.linear(f"{p}.mlp.fc2", mlp, hidden)
        inv.layer_norm(f"{enc}.norm", hidden)
        inv.linear("head.head", hidden, classes)
    return inv.items


def inventory(kind: str, size: str):
    if kind == "det":
        return detector_inventory(size)
    if kind == "rec":
        return recognizer_inventory(size)
    raise ValueError(f"unknown model kind {kind!r}")


def expected_tensor_count(kind: str, size: str) -> int:
    return (DETECTOR_TENSORS if kind == "det" else RECOGNIZER_TENSORS)[size]
