"""Adds a 16-bit PCM soundtrack to a video-only MP4 (ISO base media file format), so a
render ships as one file with sound -- the reference muxes video and audio into one mp4 with
PyAV (src/inference/render.py:193-197); no muxer is installed here, and OpenCV writes video
only.

The input MP4 keeps its bytes up to its `moov` box (so the video track's chunk offsets stay
valid); after them come a new `mdat` holding the interleaved little-endian PCM frames and a
rewritten `moov`: the original movie header with the next track id advanced, the original
tracks, and one audio track whose sample entry is `sowt` (little-endian linear PCM), one PCM
frame (all channels) per sample, all samples in one chunk.
"""
import struct
from typing import List, Tuple

import numpy as np


def _box(kind: bytes, payload: bytes) -> bytes:
    return struct.pack(">I", 8 + len(payload)) + kind + payload


def _full(kind: bytes, version: int, flags: int, payload: bytes) -> bytes:
    return _box(kind, struct.pack(">I", (version << 24) | flags) + payload)


def boxes(data: bytes, start: int = 0, end: int = None) -> List[Tuple[bytes, int, int]]:
    """(type, offset, size) of the boxes laid end to end in data[start:end]."""
    end = len(data) if end is None else end
    out, pos = [], start
    while pos + 8 <= end:
        size, kind = struct.unpack(">I4s", data[pos:pos + 8])
        if size == 1:
            size = struct.unpack(">Q", data[pos + 8:pos + 16])[0]
        elif size == 0:
            size = end - pos
        if size < 8 or pos + size > end:
            raise ValueError(f"malformed MP4 box {kind!r} at {pos}")
        out.append((kind, pos, size))
        pos += size
    return out


def _identity_matrix() -> bytes:
    return struct.pack(">9I", 0x00010000, 0, 0, 0, 0x00010000, 0, 0, 0, 0x40000000)


def _audio_trak(track_id: int, movie_timescale: int, rate: int, channels: int, frames: int,
                data_offset: int) -> bytes:
    movie_duration = frames * movie_timescale // rate
    tkhd = _full(b"tkhd", 0, 0x7, struct.pack(">IIIII", 0, 0, track_id, 0, movie_duration)
                 + b"\0" * 8 + struct.pack(">hhhh", 0, 1, 0x0100, 0) + _identity_matrix()
                 + struct.pack(">II", 0, 0))
    mdhd = _full(b"mdhd", 0, 0, struct.pack(">IIIIHH", 0, 0, rate, frames, 0x55C4, 0))  # 'und'
    hdlr = _full(b"hdlr", 0, 0, struct.pack(">I4s3I", 0, b"soun", 0, 0, 0) + b"SoundHandler\0")
    smhd = _full(b"smhd", 0, 0, struct.pack(">hH", 0, 0))
    dref = _full(b"dref", 0, 0, struct.pack(">I", 1) + _full(b"url ", 0, 1, b""))
    sowt = _box(b"sowt", b"\0" * 6 + struct.pack(">H", 1) + struct.pack(">II", 0, 0)
                + struct.pack(">HHHHI", channels, 16, 0, 0, rate << 16))
    stsd = _full(b"stsd", 0, 0, struct.pack(">I", 1) + sowt)
    stts = _full(b"stts", 0, 0, struct.pack(">III", 1, frames, 1))
    stsc = _full(b"stsc", 0, 0, struct.pack(">IIII", 1, 1, frames, 1))
    stsz = _full(b"stsz", 0, 0, struct.pack(">II", 2 * channels, frames))
    if data_offset < 2 ** 32:
        chunks = _full(b"stco", 0, 0, struct.pack(">II", 1, data_offset))
    else:
        chunks = _full(b"co64", 0, 0, struct.pack(">IQ", 1, data_offset))
    stbl = _box(b"stbl", stsd + stts + stsc + stsz + chunks)
    minf = _box(b"minf", smhd + _box(b"dinf", dref) + stbl)
    return _box(b"trak", tkhd + _box(b"mdia", mdhd + hdlr + minf))


def add_pcm_track(video_mp4: bytes, pcm: np.ndarray, rate: int) -> bytes:
    """video_mp4: the bytes of an MP4 whose `moov` is its last top-level box; pcm: int16
    [frames, channels]. Returns the bytes of the muxed file."""
    pcm = np.ascontiguousarray(pcm, dtype="<i2")
    if pcm.ndim != 2:
        raise ValueError("pcm must be [frames, channels]")
    top = boxes(video_mp4)
    if not top or top[-1][0] != b"moov":
        raise ValueError("the video MP4 must end with its moov box")
    _, moov_at, moov_size = top[-1]
    kids = boxes(video_mp4, moov_at + 8, moov_at + moov_size)
    mvhd = next(((o, s) for k, o, s in kids if k == b"mvhd"), None)
    if mvhd is None:
        raise ValueError("moov has no mvhd")
    o, s = mvhd
    raw = bytearray(video_mp4[o:o + s])
    version = raw[8]
    ts_at, dur_at, dur_fmt = (28, 32, ">Q") if version == 1 else (20, 24, ">I")
    timescale = struct.unpack(">I", raw[ts_at:ts_at + 4])[0]
    next_id = struct.unpack(">I", raw[-4:])[0]
    frames, channels = pcm.shape
    audio_duration = frames * timescale // rate
    old = struct.unpack(dur_fmt, raw[dur_at:dur_at + struct.calcsize(dur_fmt)])[0]
    raw[dur_at:dur_at + struct.calcsize(dur_fmt)] = struct.pack(dur_fmt, max(old, audio_duration))
    raw[-4:] = struct.pack(">I", next_id + 1)
    payload = pcm.tobytes()
    mdat = _box(b"mdat", payload) if len(payload) + 8 < 2 ** 32 else \
        struct.pack(">I4sQ", 1, b"mdat", 16 + len(payload)) + payload
    data_offset = moov_at + (len(mdat) - len(payload))
    others = b"".join(video_mp4[ko:ko + ks] for kk, ko, ks in kids if kk != b"mvhd")
    trak = _audio_trak(next_id, timescale, rate, channels, frames, data_offset)
    return video_mp4[:moov_at] + mdat + _box(b"moov", bytes(raw) + others + trak)


def track_handlers(mp4: bytes) -> List[bytes]:
    """Handler types ('vide', 'soun', ...) of the tracks of an MP4, in order."""
    top = {k: (o, s) for k, o, s in boxes(mp4)}
    o, s = top[b"moov"]
    out = []
    for kind, to, ts in boxes(mp4, o + 8, o + s):
        if kind != b"trak":
            continue
        mdia = next((mo, ms) for k, mo, ms in boxes(mp4, to + 8, to + ts) if k == b"mdia")
        hdlr = next((ho, hs) for k, ho, hs in boxes(mp4, mdia[0] + 8, mdia[0] + mdia[1]) if k == b"hdlr")
        out.append(mp4[hdlr[0] + 16:hdlr[0] + 20])
    return out
