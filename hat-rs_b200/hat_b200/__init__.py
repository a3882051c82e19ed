"""Python host side of the B200 HAT backend: a ctypes binding of `libhat_b200.so`.

The class `B200` mirrors the reference's `Backend` trait (src/backend.rs:29-36):
`name()` and `forward(h, w, input)` taking a planar `[3][h][w]` float32 image in
[0, 1] and returning `[3][h*scale][w*scale]`. Errors come back as `HatError`
carrying the library's code and message, the way the reference returns
`Result<_, String>`.

There is no fallback: if the CUDA library cannot be loaded, or the device cannot be
brought up, construction raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libhat_b200.so"

MODE_PARITY = 0
MODE_FAST = 1
MODE_SIMT = 2  # kernel-level calls only: the CUDA-core fp32 kernels

E_INVAL, E_IO, E_CUDA, E_NOMEM, E_SELFTEST = 1, 2, 3, 4, 5


class HatError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


SHARD_BATCH, SHARD_STRIP = 0, 1


class Opts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("mode", ctypes.c_int), ("use_graph", ctypes.c_int),
                ("simt_only", ctypes.c_int), ("ngpus", ctypes.c_int), ("devices", ctypes.POINTER(ctypes.c_int)),
                ("shard", ctypes.c_int), ("timeout_ms", ctypes.c_int)]


class Info(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_int), ("window", ctypes.c_int), ("owin", ctypes.c_int),
                ("embed", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("mlp_ratio", ctypes.c_int), ("compressed", ctypes.c_int),
                ("squeezed", ctypes.c_int), ("head_feat", ctypes.c_int),
                ("n_stages", ctypes.c_int), ("n_blocks", ctypes.c_int),
                ("conv_scale", ctypes.c_float), ("img_range", ctypes.c_float),
                ("mean", ctypes.c_float * 3), ("variant", ctypes.c_char * 32)]

    def as_dict(self) -> dict:
        d = {k: getattr(self, k) for k, _ in self._fields_}
        d["mean"] = list(self.mean)
        d["variant"] = self.variant.decode()
        return d


# Every symbol the C header declares, with its ctypes signature.
_P, _I, _F, _S, _C = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_char_p
SIGNATURES = {
    "hat_b200_create": (_I, [_C, ctypes.POINTER(Opts), ctypes.POINTER(_P), _C, _S]),
    "hat_b200_destroy": (None, [_P]),
    "hat_b200_get_info": (_I, [_P, ctypes.POINTER(Info)]),
    "hat_b200_forward": (_I, [_P, _I, _I, _I, _P, _P, _C, _S]),
    "hat_b200_forward_device": (_I, [_P, _I, _I, _I, _P, _P, _P, _C, _S]),
    "hat_b200_footprint_bytes": (_S, [_P, _I, _I]),
    "hat_b200_check_memory": (_I, [_P, _I, _I, _C, _S]),
    "hat_b200_free_vram": (_I, [_I, ctypes.POINTER(_S), ctypes.POINTER(_S)]),
    "hat_b200_probe": (_I, []),
    "hat_b200_selftest": (_I, [_I, _C, _S]),
    "hat_b200_inspect": (_I, [_C, ctypes.POINTER(Info), _C, _S]),
    "hat_b200_linear": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _P]),
    "hat_b200_conv3x3": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "hat_b200_window_attention": (_I, [_I, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "hat_b200_overlap_attention": (_I, [_I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "hat_b200_linear_noalloc": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _P, _C, _S]),
    "hat_b200_strip_rows": (_I, [_I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "hat_b200_forward_tiled": (_I, [_P, _I, _I, _P, _P, _I, _I, _P, _C, _S]),
    "hat_b200_auto_tile": (_I, [_I, _I, _I, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _I,
                                ctypes.POINTER(_I)]),
    "hat_b200_gpu_auto_tile": (_I, [_P, _I, _I, ctypes.POINTER(_I), _C, _S]),
    "hat_b200_nccl_unique_id": (_I, [_P, _S, _C, _S]),
    "hat_b200_attach_strip": (_I, [_P, _I, _I, _P, _S, _C, _S]),
    "hat_b200_launch_count": (ctypes.c_uint64, [_P]),
    "hat_b200_profile": (_I, [_P, _I, _I, _C, _S, _C, _S]),
    "hat_b200_sync": (_I, [_P, _C, _S]),
    "hat_b200_fp16_pairs": (_I, [_P]),
    "hat_b200_gpu_count": (_I, [_P]),
    "hat_b200_set_timeout": (_I, [_P, _I]),
    "hat_b200_png_load": (_I, [_C, _P, _S, ctypes.POINTER(_I), ctypes.POINTER(_I), _C, _S]),
    "hat_b200_png_decode": (_I, [_P, _S, _P, _S, ctypes.POINTER(_I), ctypes.POINTER(_I), _C, _S]),
    "hat_b200_to_rgb8": (_I, [_P, _I, _I, _P]),
    "hat_b200_png_save": (_I, [_C, _I, _I, _P, _C, _S]),
    "hat_b200_png_encode": (_I, [_I, _I, _P, _P, _S, ctypes.POINTER(_S), _C, _S]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (built on demand when the .so is missing)."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            from . import build as _b
            _b.build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _err():
    return ctypes.create_string_buffer(4096)


def _check(rc: int, buf) -> None:
    if rc != 0:
        raise HatError(rc, buf.value.decode(errors="replace"))


def inspect(path: str) -> dict:
    """Read and validate a checkpoint without a device (src/weights.rs:60-265)."""
    info, e = Info(), _err()
    _check(lib().hat_b200_inspect(str(path).encode(), ctypes.byref(info), e, len(e)), e)
    return info.as_dict()


def probe() -> bool:
    return bool(lib().hat_b200_probe())


def free_vram(device: int = 0):
    f, t = ctypes.c_size_t(), ctypes.c_size_t()
    rc = lib().hat_b200_free_vram(device, ctypes.byref(f), ctypes.byref(t))
    if rc:
        raise HatError(rc, f"free_vram: device {device} unavailable")
    return f.value, t.value


def selftest(device: int = 0):
    """`--cuda-selftest`: (passed, report)."""
    buf = ctypes.create_string_buffer(1 << 16)
    rc = lib().hat_b200_selftest(device, buf, len(buf))
    return rc == 0, buf.value.decode(errors="replace")


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class B200:
    """The B200 backend behind the reference's `Backend` contract."""

    def __init__(self, path: str, device: int = 0, mode: int = MODE_PARITY, use_graph: bool = True,
                 simt_only: bool = False, devices=None, shard: int = SHARD_BATCH, timeout_ms: int = 0):
        """`devices`: a list of CUDA ordinals for one handle over several GPUs, whose
        `forward` splits its work as `shard` says (SHARD_BATCH: the images; SHARD_STRIP:
        every image's rows, NCCL halo exchange between the GPUs)."""
        self._h = ctypes.c_void_p()
        opts = Opts(device, mode, int(use_graph), int(simt_only))
        if devices is not None and len(devices) > 1:
            self._devs = (ctypes.c_int * len(devices))(*devices)
            opts.ngpus = len(devices)
            opts.devices = self._devs
            opts.device = devices[0]
            opts.shard = shard
        opts.timeout_ms = timeout_ms
        e = _err()
        _check(lib().hat_b200_create(str(path).encode(), ctypes.byref(opts), ctypes.byref(self._h), e,
                                     len(e)), e)
        info = Info()
        lib().hat_b200_get_info(self._h, ctypes.byref(info))
        self.info = info.as_dict()
        self.scale = self.info["scale"]
        self.device = device

    def close(self):
        if self._h:
            lib().hat_b200_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def name() -> str:
        return "b200"

    def forward(self, h: int, w: int, image: np.ndarray) -> np.ndarray:
        """Backend::forward: planar `[3][h][w]` → `[3][h*s][w*s]` (host arrays)."""
        return self.forward_batch(np.asarray(image, np.float32).reshape(1, 3, h, w))[0]

    def forward_batch(self, images: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(images, dtype=np.float32)
        n, ch, h, w = x.shape
        if ch != 3:
            raise HatError(E_INVAL, f"expected 3 channels, got {ch}")
        s = self.scale
        out = np.empty((n, 3, h * s, w * s), np.float32)
        e = _err()
        _check(lib().hat_b200_forward(self._h, n, h, w, _ptr(x), _ptr(out), e, len(e)), e)
        return out

    def forward_device(self, d_in: int, d_out: int, n: int, h: int, w: int, stream: int = 0) -> None:
        """Enqueue a pass on device pointers (`int` addresses) on `stream`."""
        e = _err()
        _check(lib().hat_b200_forward_device(self._h, n, h, w, ctypes.c_void_p(d_in),
                                             ctypes.c_void_p(d_out), ctypes.c_void_p(stream), e,
                                             len(e)), e)

    def forward_tiled(self, h: int, w: int, image: np.ndarray, tile: int, margin: int):
        """tile::forward: `--tile` / `--mem` cores with a margin of context; returns
        (planar output, tiling info dict)."""
        x = np.ascontiguousarray(image, dtype=np.float32).reshape(3, h, w)
        out = np.empty((3, h * self.scale, w * self.scale), np.float32)
        info, e = Tiling(), _err()
        _check(lib().hat_b200_forward_tiled(self._h, h, w, _ptr(x), _ptr(out), tile, margin, ctypes.byref(info),
                                            e, len(e)), e)
        return out, info.as_dict()

    def gpu_auto_tile(self, h: int, w: int) -> int:
        t, e = _I(), _err()
        _check(lib().hat_b200_gpu_auto_tile(self._h, h, w, ctypes.byref(t), e, len(e)), e)
        return t.value

    def attach_strip(self, rank: int, nranks: int, uid: bytes) -> None:
        """Shard every later pass over `nranks` GPUs by row strips (collective: all ranks
        call it with the same NCCL unique id); each pass then writes this rank's rows."""
        e = _err()
        _check(lib().hat_b200_attach_strip(self._h, rank, nranks, uid, len(uid), e, len(e)), e)

    def sync(self) -> None:
        """Wait for this handle's device work; raise if a kernel flagged an error."""
        e = _err()
        _check(lib().hat_b200_sync(self._h, e, len(e)), e)

    def set_timeout(self, ms: int) -> None:
        """Deadline of a strip-sharded call's device work (0: the 120 s default)."""
        lib().hat_b200_set_timeout(self._h, ms)

    def gpu_count(self) -> int:
        return int(lib().hat_b200_gpu_count(self._h))

    def fp16_pairs(self) -> bool:
        """Parity-mode operands are fp16 pairs (False: tf32 pairs, or another mode)."""
        return bool(lib().hat_b200_fp16_pairs(self._h))

    def footprint_bytes(self, h: int, w: int) -> int:
        return int(lib().hat_b200_footprint_bytes(self._h, h, w))

    def check_memory(self, h: int, w: int) -> None:
        e = _err()
        _check(lib().hat_b200_check_memory(self._h, h, w, e, len(e)), e)

    def launch_count(self) -> int:
        return int(lib().hat_b200_launch_count(self._h))

    def profile(self, h: int, w: int) -> dict:
        """Per-kind device time of one eager pass: {kind: {launches, ms, flops, bytes}}."""
        import json
        buf, e = ctypes.create_string_buffer(1 << 16), _err()
        _check(lib().hat_b200_profile(self._h, h, w, buf, len(buf), e, len(e)), e)
        return json.loads(buf.value.decode())


# Kernel-level calls on device pointers (ints), the units --cuda-selftest checks.
def linear(mode, x, w, b, y, m, n, k, stream=0):
    rc = lib().hat_b200_linear(mode, x, w, b, y, m, n, k, stream)
    if rc:
        raise HatError(rc, "linear launch failed")


class Tiling(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("tile", "margin", "scale", "tiles", "largest_h", "largest_w")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


def auto_tile(h: int, w: int, win: int, budget_bytes: int, per_pixel_floats: int, constant_floats: int,
              margin: int):
    """tile::auto_tile: the core side for a memory budget, or None when one window does not fit."""
    t = _I()
    rc = lib().hat_b200_auto_tile(h, w, win, budget_bytes, per_pixel_floats, constant_floats, margin,
                                  ctypes.byref(t))
    if rc == E_NOMEM:
        return None
    if rc:
        raise HatError(rc, "auto_tile: bad arguments")
    return t.value


def strip_rows(height: int, nranks: int, rank: int):
    """Padded rows [r0, r1) of rank `rank`'s strip (window-aligned, as equal as possible)."""
    r0, r1 = _I(), _I()
    rc = lib().hat_b200_strip_rows(height, nranks, rank, ctypes.byref(r0), ctypes.byref(r1))
    if rc:
        raise HatError(rc, f"no strip plan for {height} rows over {nranks} ranks")
    return r0.value, r1.value


def nccl_unique_id() -> bytes:
    """An NCCL unique id for hat_b200_attach_strip (made on one rank, shared with all)."""
    buf, e = ctypes.create_string_buffer(128), _err()
    _check(lib().hat_b200_nccl_unique_id(buf, 128, e, len(e)), e)
    return buf.raw


def linear_noalloc(mode, x, w, b, y, m, n, k, stream=0):
    """`linear` with all scratch in the library's fixed device array (no allocation);
    sizes beyond NOALLOC_SCRATCH_BYTES raise HatError(EINVAL)."""
    e = _err()
    _check(lib().hat_b200_linear_noalloc(mode, x, w, b, y, m, n, k, stream, e, len(e)), e)


NOALLOC_SCRATCH_BYTES = 8 << 20


def conv3x3(mode, x, w, b, y, hgt, wid, cin, cout, stream=0):
    rc = lib().hat_b200_conv3x3(mode, x, w, b, y, hgt, wid, cin, cout, stream)
    if rc:
        raise HatError(rc, "conv3x3 launch failed")


def window_attention(mode, qkv, table, out, hp, wp, c, heads, shift, stream=0):
    rc = lib().hat_b200_window_attention(mode, qkv, table, out, hp, wp, c, heads, shift, stream)
    if rc:
        raise HatError(rc, "window attention launch failed")


def overlap_attention(mode, qkv, table, out, hp, wp, c, heads, stream=0):
    rc = lib().hat_b200_overlap_attention(mode, qkv, table, out, hp, wp, c, heads, stream)
    if rc:
        raise HatError(rc, "overlap attention launch failed")


# PNG file I/O around the forward pass (src/image.rs).
def png_load(path: str) -> np.ndarray:
    """image::load_rgb: a PNG file as planar `[3][h][w]` float32 in [0, 1]."""
    w, h, e = _I(), _I(), _err()
    _check(lib().hat_b200_png_load(str(path).encode(), None, 0, ctypes.byref(w), ctypes.byref(h), e, len(e)), e)
    out = np.empty((3, h.value, w.value), np.float32)
    _check(lib().hat_b200_png_load(str(path).encode(), _ptr(out), out.size, ctypes.byref(w), ctypes.byref(h), e,
                                   len(e)), e)
    return out


def png_decode(data: bytes) -> np.ndarray:
    """image::load_rgb_stream: PNG bytes as planar `[3][h][w]` float32 in [0, 1]."""
    buf = (ctypes.c_uint8 * len(data)).from_buffer_copy(data)
    w, h, e = _I(), _I(), _err()
    _check(lib().hat_b200_png_decode(buf, len(data), None, 0, ctypes.byref(w), ctypes.byref(h), e, len(e)), e)
    out = np.empty((3, h.value, w.value), np.float32)
    _check(lib().hat_b200_png_decode(buf, len(data), _ptr(out), out.size, ctypes.byref(w), ctypes.byref(h), e,
                                     len(e)), e)
    return out


def to_rgb8(planar: np.ndarray) -> np.ndarray:
    """Image::to_rgb8: planar `[3][h][w]` float to interleaved `[h][w][3]` uint8."""
    x = np.ascontiguousarray(planar, np.float32)
    _, h, w = x.shape
    out = np.empty((h, w, 3), np.uint8)
    rc = lib().hat_b200_to_rgb8(_ptr(x), w, h, _ptr(out))
    if rc:
        raise HatError(rc, "to_rgb8: bad arguments")
    return out


def png_save(path: str, rgb: np.ndarray) -> None:
    """image::save_rgb: interleaved `[h][w][3]` uint8 to a PNG file."""
    x = np.ascontiguousarray(rgb, np.uint8)
    h, w, _ = x.shape
    e = _err()
    _check(lib().hat_b200_png_save(str(path).encode(), w, h, _ptr(x), e, len(e)), e)


def png_encode(rgb: np.ndarray) -> bytes:
    """image::save_rgb_stream: interleaved `[h][w][3]` uint8 to PNG bytes."""
    x = np.ascontiguousarray(rgb, np.uint8)
    h, w, _ = x.shape
    n, e = _S(), _err()
    lib().hat_b200_png_encode(w, h, _ptr(x), None, 0, ctypes.byref(n), e, len(e))
    out = (ctypes.c_uint8 * n.value)()
    _check(lib().hat_b200_png_encode(w, h, _ptr(x), out, n.value, ctypes.byref(n), e, len(e)), e)
    return bytes(out)[:n.value]
