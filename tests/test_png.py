"""PNG file I/O (src/image.rs of the reference) through the C ABI, on the CPU.

The files are made here by an independent writer that follows the PNG specification with
Python's zlib: every colour type the reference decodes (grey, grey + alpha, RGB, RGBA) at 8
and 16 bits, every row filter, Adam7 interlacing, image data split over several IDAT
chunks. The expected planar floats follow src/image.rs:55-96 (sample / 255 or / 65535, grey
replicated, alpha dropped). The encoder's files are read back by an independent decoder
here, and the refusals match the reference's (indexed colour, bit depths other than 8/16).
"""
import struct
import zlib

import numpy as np
import pytest

import hat_b200

CHANNELS = {0: 1, 4: 2, 2: 3, 6: 4}
ADAM7 = [(0, 0, 8, 8), (4, 0, 8, 8), (0, 4, 4, 8), (2, 0, 4, 4), (0, 2, 2, 4), (1, 0, 2, 2), (0, 1, 1, 2)]


def _chunk(t, body):
    return struct.pack(">I", len(body)) + t + body + struct.pack(">I", zlib.crc32(t + body) & 0xFFFFFFFF)


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
    return a if pa <= pb and pa <= pc else (b if pb <= pc else c)


def _filter_rows(raw, bpp, rng):
    """Filter each row of `raw` ([rows][rowbytes] uint8) with a random filter type."""
    out = bytearray()
    prev = np.zeros(raw.shape[1], np.int64)
    for row in raw.astype(np.int64):
        ft = int(rng.integers(0, 5))
        f = np.empty_like(row)
        for i in range(len(row)):
            a = row[i - bpp] if i >= bpp else 0
            b = prev[i]
            c = prev[i - bpp] if i >= bpp else 0
            pred = [0, a, b, (a + b) >> 1, _paeth(a, b, c)][ft]
            f[i] = (row[i] - pred) & 0xFF
        out.append(ft)
        out += bytes(f.astype(np.uint8))
        prev = row
    return bytes(out)


def _write_png(px, depth, ctype, interlace=False, idat_parts=3, seed=0):
    """px: [h][w][channels] integer samples."""
    h, w, ch = px.shape
    rng = np.random.default_rng(seed)
    bps = depth // 8
    def raw_of(sub):
        if depth == 16:
            b = sub.astype(">u2").view(np.uint8)
        else:
            b = sub.astype(np.uint8)
        return b.reshape(sub.shape[0], -1)
    if not interlace:
        data = _filter_rows(raw_of(px), ch * bps, rng)
    else:
        data = b""
        for x0, y0, dx, dy in ADAM7:
            sub = px[y0::dy, x0::dx]
            if sub.shape[0] and sub.shape[1]:
                data += _filter_rows(raw_of(sub), ch * bps, rng)
    z = zlib.compress(data, 9)
    cut = [len(z) * i // idat_parts for i in range(idat_parts + 1)]
    ihdr = struct.pack(">IIBBBBB", w, h, depth, ctype, 0, 0, int(interlace))
    out = b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", ihdr)
    out += _chunk(b"tEXt", b"Comment\x00made by the test")
    for i in range(idat_parts):
        out += _chunk(b"IDAT", z[cut[i]:cut[i + 1]])
    return out + _chunk(b"IEND", b"")


def _expected(px, depth):
    scale = np.float32(1.0 / 255.0) if depth == 8 else np.float32(1.0 / 65535.0)
    v = px.astype(np.float32) * scale
    rgb = np.repeat(v[..., :1], 3, axis=2) if px.shape[2] <= 2 else v[..., :3]
    return np.ascontiguousarray(rgb.transpose(2, 0, 1))


@pytest.mark.parametrize("ctype", [0, 4, 2, 6])
@pytest.mark.parametrize("depth", [8, 16])
@pytest.mark.parametrize("interlace", [False, True])
def test_decode_matches_the_specification(ctype, depth, interlace, tmp_path):
    rng = np.random.default_rng(ctype * 100 + depth + interlace)
    h, w = 13, 11  # not multiples of 8: partial Adam7 passes
    px = rng.integers(0, 1 << depth, (h, w, CHANNELS[ctype]))
    data = _write_png(px, depth, ctype, interlace, seed=depth + ctype)
    want = _expected(px, depth)
    got = hat_b200.png_decode(data)
    assert got.shape == (3, h, w)
    assert np.array_equal(got, want)
    p = tmp_path / "x.png"
    p.write_bytes(data)
    assert np.array_equal(hat_b200.png_load(p), want)


def _read_png_rgb8(data):
    """Independent decoder for the encoder's output (8-bit RGB, not interlaced)."""
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    pos, z, hdr = 8, b"", None
    while pos < len(data):
        n, t = struct.unpack(">I4s", data[pos:pos + 8])
        body = data[pos + 8:pos + 8 + n]
        assert struct.unpack(">I", data[pos + 8 + n:pos + 12 + n])[0] == zlib.crc32(t + body) & 0xFFFFFFFF
        if t == b"IHDR":
            hdr = struct.unpack(">IIBBBBB", body)
        elif t == b"IDAT":
            z += body
        pos += 12 + n
    w, h, depth, ctype, _, _, il = hdr
    assert (depth, ctype, il) == (8, 2, 0)
    raw = zlib.decompress(z)
    rb = w * 3
    out = np.zeros((h, rb), np.int64)
    prev = np.zeros(rb, np.int64)
    for y in range(h):
        ft, row = raw[y * (rb + 1)], np.frombuffer(raw[y * (rb + 1) + 1:(y + 1) * (rb + 1)], np.uint8).astype(np.int64)
        cur = np.zeros(rb, np.int64)
        for i in range(rb):
            a = cur[i - 3] if i >= 3 else 0
            b, c = prev[i], (prev[i - 3] if i >= 3 else 0)
            cur[i] = (row[i] + [0, a, b, (a + b) >> 1, _paeth(a, b, c)][ft]) & 0xFF
        out[y], prev = cur, cur
    return out.reshape(h, w, 3).astype(np.uint8)


def test_encode_reads_back(tmp_path):
    rng = np.random.default_rng(5)
    rgb = rng.integers(0, 256, (17, 23, 3)).astype(np.uint8)
    data = hat_b200.png_encode(rgb)
    assert np.array_equal(_read_png_rgb8(data), rgb)
    p = tmp_path / "o.png"
    hat_b200.png_save(p, rgb)
    assert p.read_bytes() == data
    # and through the library's own decoder: the planar floats of the same bytes
    back = hat_b200.png_load(p)
    assert np.array_equal(back, rgb.transpose(2, 0, 1).astype(np.float32) * np.float32(1 / 255))


def test_to_rgb8_clamps_and_rounds_like_the_reference():
    # Image::to_rgb8 (src/image.rs:29-39): clamp to [0, 1], x 255, floor(v + 0.5), min 255;
    # NaN becomes 255 (f32::min returns the other operand).
    v = np.array([-1.0, 0.0, 0.5 / 255, 0.49 / 255, 1.5 / 255, 0.5, 1.0, 7.0, np.nan, np.inf, -np.inf, 0.9999],
                 np.float32)
    planar = np.stack([v, v[::-1], np.roll(v, 3)])[:, None, :]
    got = hat_b200.to_rgb8(planar)[0]
    def ref(x):
        if np.isnan(x):
            return 255
        y = np.float32(min(max(x, np.float32(0)), np.float32(1))) * np.float32(255)
        return int(min(np.floor(y + np.float32(0.5)), 255.0))
    want = np.array([[ref(planar[c, 0, i]) for c in range(3)] for i in range(len(v))], np.uint8)
    assert np.array_equal(got, want)


def test_refusals(tmp_path):
    px = np.zeros((4, 4, 1), np.int64)
    good = _write_png(px, 8, 0)
    # indexed colour: the reference refuses it
    ihdr = struct.pack(">IIBBBBB", 4, 4, 8, 3, 0, 0, 0)
    indexed = good[:8] + _chunk(b"IHDR", ihdr) + good[8 + 25:]
    with pytest.raises(hat_b200.HatError, match="colour type Indexed") as e:
        hat_b200.png_decode(indexed)
    assert e.value.code == hat_b200.E_IO
    with pytest.raises(hat_b200.HatError, match="bit depth"):
        hat_b200.png_decode(good[:8] + _chunk(b"IHDR", struct.pack(">IIBBBBB", 4, 4, 4, 0, 0, 0, 0)) + good[33:])
    bad_crc = bytearray(good)
    bad_crc[30] ^= 0xFF
    with pytest.raises(hat_b200.HatError, match="CRC"):
        hat_b200.png_decode(bytes(bad_crc))
    with pytest.raises(hat_b200.HatError):
        hat_b200.png_decode(good[:40])
    with pytest.raises(hat_b200.HatError, match="signature"):
        hat_b200.png_decode(b"GIF89a" + good[6:])
    with pytest.raises(hat_b200.HatError) as e:
        hat_b200.png_load(tmp_path / "missing.png")
    assert e.value.code == hat_b200.E_IO
