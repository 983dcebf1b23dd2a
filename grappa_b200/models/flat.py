"""Flat parameter storage shared by the torch modules and the sm_100a engine.

Every parameter of a model lives in one fp32 buffer laid out the way the GEMM
kernels consume it: each weight matrix is a [rows, cols] row-major segment whose
row stride is padded to a multiple of 8 elements (16 bytes, the TMA stride rule)
and whose unused pad entries stay zero.  The modules' ``nn.Parameter`` objects
are views into that buffer, so ``state_dict`` keeps the reference's key names and
shapes (DGL 1.x conventions) while the engine's fused Adam, the split-K gradient
reductions and the bf16 working copy all address the same flat layout.
"""
import math

import torch
from torch import nn


def pad8(n):
    return (int(n) + 7) // 8 * 8


class Segment:
    def __init__(self, name, rows, cols, offset):
        self.name, self.rows, self.cols, self.offset = name, rows, cols, offset

    @property
    def numel(self):
        return self.rows * self.cols

    def view(self, flat):
        return flat[self.offset:self.offset + self.numel].view(self.rows, self.cols)


class FlatModule(nn.Module):
    """Base class of the GNN models: owns the flat buffer and re-binds the views."""

    def __init__(self):
        super().__init__()
        self._segments = {}
        self._bindings = []  # (module, attr, segment name, rows, cols, transpose, shape)
        self._size = 0
        self.flat = None

    # --- layout -------------------------------------------------------------------------
    def add_segment(self, name, rows, cols):
        cols = pad8(cols)
        seg = Segment(name, int(rows), cols, self._size)
        self._segments[name] = seg
        self._size += seg.numel
        self._size = (self._size + 63) // 64 * 64  # 256-byte aligned segments
        return seg

    def bind(self, module, attr, seg_name, rows, cols, transpose=False, shape=None):
        """module.attr = segment[rows, cols] (a view); ``rows``/``cols`` are slices or
        indices, ``shape`` optionally reshapes the (contiguous) view."""
        self._bindings.append((module, attr, seg_name, rows, cols, transpose, shape))

    def _view(self, flat, seg_name, rows, cols, transpose, shape):
        v = self._segments[seg_name].view(flat)[rows, cols]
        if transpose:
            v = v.t()
        if shape is not None:
            v = v.view(shape)
        return v

    def segment(self, name):
        return self._segments[name]

    def layer_buckets(self, n_layers):
        """[(lo, hi)] element range of every layer's parameters (segments named
        ``layers.{i}.*`` or ``batch_norms.{i}``) in the flat buffer, or None when a layer's
        segments are not contiguous.  Ranges start on 64-element boundaries."""
        import re

        spans = {}
        for name, seg in self._segments.items():
            m = re.match(r"^(?:layers|batch_norms)\.(\d+)(?:\.|$)", name)
            if m is None:
                return None
            i = int(m.group(1))
            end = (seg.offset + seg.numel + 63) // 64 * 64
            lo, hi, total = spans.get(i, (seg.offset, end, 0))
            spans[i] = (min(lo, seg.offset), max(hi, end), total + (end - seg.offset))
        if sorted(spans) != list(range(n_layers)):
            return None
        out = []
        for i in range(n_layers):
            lo, hi, total = spans[i]
            if hi - lo != total:
                return None  # another layer's segment lies inside this layer's range
            out.append((lo, hi))
        return out

    def finalize(self, init_fn, device="cpu"):
        flat = torch.zeros(self._size, dtype=torch.float32, device=device)
        self._rebind(flat)
        with torch.no_grad():
            init_fn()

    def _rebind(self, flat):
        self.flat = flat
        for module, attr, seg_name, rows, cols, transpose, shape in self._bindings:
            v = self._view(flat, seg_name, rows, cols, transpose, shape)
            if attr in module._parameters:
                del module._parameters[attr]
            module.register_parameter(attr, nn.Parameter(v))

    def place(self, device):
        """Move the flat buffer (and the buffers) to ``device`` and re-bind every view."""
        device = torch.device(device)
        if self.flat is not None and self.flat.device != device:
            self._rebind(self.flat.to(device))
        for m in self.modules():
            for k, b in list(m._buffers.items()):
                if b is not None and b.device != device:
                    m._buffers[k] = b.to(device)
        return self

    @property
    def num_flat(self):
        return self._size

    def flat_grad(self):
        """Allocate a flat fp32 gradient buffer and make every ``param.grad`` a view of it."""
        g = torch.zeros_like(self.flat)
        for module, attr, seg_name, rows, cols, transpose, shape in self._bindings:
            p = module._parameters.get(attr)
            if p is None:
                continue
            p.grad = self._view(g, seg_name, rows, cols, transpose, shape)
        return g

    def state_dict_contiguous(self):
        """state_dict with standalone contiguous tensors (what gets saved in checkpoints)."""
        return {k: v.detach().clone().contiguous() for k, v in self.state_dict().items()}

    def load_state_dict(self, state_dict, strict=True):
        # copy into the existing views so that the flat layout is preserved
        own = self.state_dict(keep_vars=True)
        missing = [k for k in own if k not in state_dict]
        unexpected = [k for k in state_dict if k not in own]
        if strict and (missing or unexpected):
            raise RuntimeError(f"state_dict mismatch: missing={missing} unexpected={unexpected}")
        with torch.no_grad():
            for k, v in state_dict.items():
                if k in own:
                    own[k].copy_(v.to(own[k].device, own[k].dtype))
        return nn.modules.module._IncompatibleKeys(missing, unexpected)


def xavier_uniform_(t, gain=1.0):
    fan_out, fan_in = t.shape[0], t.shape[1]
    bound = gain * math.sqrt(6.0 / (fan_in + fan_out))
    with torch.no_grad():
        t.uniform_(-bound, bound)


def xavier_normal_(t, gain=1.0):
    fan_out, fan_in = t.shape[0], t.shape[1]
    std = gain * math.sqrt(2.0 / (fan_in + fan_out))
    with torch.no_grad():
        t.normal_(0.0, std)
