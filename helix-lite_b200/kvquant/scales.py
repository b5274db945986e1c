"""Calibrated nuq scales: the containers of src/kvquant/scales.py:14-140.

Same fields, shapes and ``.to / .save / .load`` file format as the reference,
so existing ``.pt`` scale files load unchanged:

* ``PerChannelScale`` (Keys):   poles (H, D, L), thresholds (H, D)
* ``PerTokenScale``  (Values):  poles (H, T_cal, L), thresholds (H, T_cal);
  positions >= T_cal reuse row T_cal - 1
* ``KVScales``: one key and one value scale per layer, plus
  ``first_few_fp16`` and ``num_bits`` metadata.

``layer_struct`` adds the device view the CUDA kernels take.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from hxlib import LayerScales


def _to(t, device):
    return t.to(device)


@dataclass
class PerChannelScale:
    poles: torch.Tensor
    upper_threshold: torch.Tensor
    lower_threshold: torch.Tensor
    num_bits: int = 2

    def to(self, device) -> "PerChannelScale":
        return PerChannelScale(_to(self.poles, device), _to(self.upper_threshold, device),
                               _to(self.lower_threshold, device), self.num_bits)


@dataclass
class PerTokenScale:
    poles: torch.Tensor
    upper_threshold: torch.Tensor
    lower_threshold: torch.Tensor
    num_bits: int = 2

    def to(self, device) -> "PerTokenScale":
        return PerTokenScale(_to(self.poles, device), _to(self.upper_threshold, device),
                             _to(self.lower_threshold, device), self.num_bits)


@dataclass
class KVScales:
    per_layer_keys: list = field(default_factory=list)
    per_layer_values: list = field(default_factory=list)
    first_few_fp16: int = 4
    num_bits: int = 2

    def __post_init__(self) -> None:
        if self.per_layer_keys and self.per_layer_values and \
                len(self.per_layer_keys) != len(self.per_layer_values):
            raise AssertionError("key and value scales must cover the same number of layers")
        self._dev_cache = {}

    @property
    def num_layers(self) -> int:
        return len(self.per_layer_keys)

    def to(self, device) -> "KVScales":
        return KVScales([s.to(device) for s in self.per_layer_keys],
                        [s.to(device) for s in self.per_layer_values],
                        self.first_few_fp16, self.num_bits)

    def _payload(self):
        def one(s):
            return {"poles": s.poles, "upper_threshold": s.upper_threshold,
                    "lower_threshold": s.lower_threshold, "num_bits": s.num_bits}
        return {"per_layer_keys": [one(s) for s in self.per_layer_keys],
                "per_layer_values": [one(s) for s in self.per_layer_values],
                "first_few_fp16": self.first_few_fp16, "num_bits": self.num_bits}

    def save(self, path: str) -> None:
        torch.save(self._payload(), path)

    @classmethod
    def load(cls, path: str, map_location="cpu") -> "KVScales":
        d = torch.load(path, map_location=map_location, weights_only=True)
        return cls([PerChannelScale(**s) for s in d["per_layer_keys"]],
                   [PerTokenScale(**s) for s in d["per_layer_values"]],
                   d["first_few_fp16"], d["num_bits"])

    # -- device view for the kernels --
    def device_layer(self, layer: int, device):
        """(LayerScales struct, tensors kept alive) for one layer on `device`.

        Poles and thresholds become contiguous fp16 on the device once and are
        cached; the reference kernels read fp16 scales too
        (src/kvquant/compact_pool.py:222-287). The code thresholds the pack
        kernel bisects (hx_scales_prepare: per codebook row, the fp16 values
        where the reference's nearest-pole scan moves to the next level) are
        computed on the device with them, once per layer and device.
        """
        dev = torch.device(device)
        key = (layer, dev.type, dev.index)
        hit = self._dev_cache.get(key)
        if hit is not None:
            return hit
        ks, vs = self.per_layer_keys[layer], self.per_layer_values[layer]

        def f16(t):
            return t.to(device=dev, dtype=torch.float16).contiguous()
        ts = [f16(ks.poles), f16(ks.upper_threshold), f16(ks.lower_threshold),
              f16(vs.poles), f16(vs.upper_threshold), f16(vs.lower_threshold)]
        H, D, levels_k = (int(x) for x in ks.poles.shape)
        t_cal, levels_v = int(vs.poles.shape[1]), int(vs.poles.shape[-1])
        st = LayerScales(*(t.data_ptr() for t in ts), levels_k, levels_v, t_cal, 0, None, None)
        if D % 2 == 0 and levels_k <= 16 and levels_v <= 16:
            from hxlib import call, ptr, stream
            kt = torch.empty((H, D // 2, 16), dtype=torch.int32, device=dev)
            vt = torch.empty((H, t_cal, 16), dtype=torch.int32, device=dev)
            with torch.cuda.device(dev):
                call("hx_scales_prepare", stream(dev), ctypes.byref(st), H, D, ptr(kt), ptr(vt))
            st.k_thresh, st.v_thresh = kt.data_ptr(), vt.data_ptr()
            ts += [kt, vt]
        hit = (st, ts)
        self._dev_cache[key] = hit
        return hit
