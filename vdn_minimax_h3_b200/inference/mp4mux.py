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


# ------------------------------------------------------------------ segment concatenation
# Video tracks encoded in parallel (one encoder per frame range, each starting with a key
# frame) are joined into one track: every segment's samples are copied, in order, into one
# mdat; the first segment's sample entry (the codec configuration, identical for segments
# written by the same encoder settings) describes them all; the sample tables are rebuilt
# with one chunk per segment and the sync-sample numbers shifted; edit lists are dropped.
_CONTAINERS = {b"moov", b"trak", b"mdia", b"minf", b"stbl", b"dinf"}


def _children(data: bytes, off: int, size: int):
    return boxes(data, off + 8, off + size)


def _find_child(data, off, size, kind):
    return next(((o, s) for k, o, s in _children(data, off, size) if k == kind), None)


def _u32s(b: bytes, n: int, at: int):
    return list(struct.unpack(f">{n}I", b[at:at + 4 * n]))


def _video_samples(data: bytes):
    """(sample byte ranges, per-sample durations, sync sample numbers, ctts offsets or
    None, media timescale) of the first video track of an MP4."""
    moov = next((o, s) for k, o, s in boxes(data) if k == b"moov")
    for kind, to, ts in _children(data, *moov):
        if kind != b"trak":
            continue
        mdia = _find_child(data, to, ts, b"mdia")
        hdlr = _find_child(data, *mdia, b"hdlr")
        if data[hdlr[0] + 16:hdlr[0] + 20] != b"vide":
            continue
        mdhd = _find_child(data, *mdia, b"mdhd")
        version = data[mdhd[0] + 8]
        at = mdhd[0] + (28 if version == 1 else 20)
        timescale = struct.unpack(">I", data[at:at + 4])[0]
        stbl = _find_child(data, *_find_child(data, *mdia, b"minf"), b"stbl")
        tab = {k: (o, s) for k, o, s in _children(data, *stbl)}
        o = tab[b"stts"][0]
        n = _u32s(data, 1, o + 12)[0]
        runs = _u32s(data, 2 * n, o + 16)
        durations = [d for c, d in zip(runs[::2], runs[1::2]) for _ in range(c)]
        o = tab[b"stsz"][0]
        fixed, count = _u32s(data, 2, o + 12)
        sizes = [fixed] * count if fixed else _u32s(data, count, o + 20)
        o = tab[b"stsc"][0]
        n = _u32s(data, 1, o + 12)[0]
        stsc = _u32s(data, 3 * n, o + 16)
        if b"stco" in tab:
            o = tab[b"stco"][0]
            n = _u32s(data, 1, o + 12)[0]
            chunks = _u32s(data, n, o + 16)
        else:
            o = tab[b"co64"][0]
            n = _u32s(data, 1, o + 12)[0]
            chunks = list(struct.unpack(f">{n}Q", data[o + 16:o + 16 + 8 * n]))
        ranges, sample = [], 0
        for c, base in enumerate(chunks, start=1):
            per = next(stsc[3 * i + 1] for i in range(len(stsc) // 3 - 1, -1, -1) if stsc[3 * i] <= c)
            pos = base
            for _ in range(per):
                ranges.append((pos, sizes[sample]))
                pos += sizes[sample]
                sample += 1
        sync = None
        if b"stss" in tab:
            o = tab[b"stss"][0]
            n = _u32s(data, 1, o + 12)[0]
            sync = _u32s(data, n, o + 16)
        ctts = None
        if b"ctts" in tab:
            o = tab[b"ctts"][0]
            n = _u32s(data, 1, o + 12)[0]
            vals = list(struct.unpack(f">{2 * n}i", data[o + 16:o + 16 + 8 * n]))
            ctts = [v for c, v in zip(vals[::2], vals[1::2]) for _ in range(c)]
        return ranges, durations, sync, ctts, timescale
    raise ValueError("no video track")


def _runs(values):
    out = []
    for v in values:
        if out and out[-1][1] == v:
            out[-1][0] += 1
        else:
            out.append([1, v])
    return out


def concat_video_segments(segments: List[bytes]) -> bytes:
    """One video-only MP4 from MP4 segments encoded with identical settings (moov last in
    each, a key frame first in each)."""
    if len(segments) == 1:
        return segments[0]
    first = segments[0]
    parsed = [_video_samples(s) for s in segments]
    timescale = parsed[0][4]
    if any(p[4] != timescale for p in parsed):
        raise ValueError("segments use different media timescales")
    ftyp = next((first[o:o + s] for k, o, s in boxes(first) if k == b"ftyp"), b"")
    payload, chunk_starts, counts = bytearray(), [], []
    durations, sync, ctts = [], [], []
    header = 16                                    # 64-bit mdat header: offsets known now
    for (ranges, dur, sy, ct, _), seg in zip(parsed, segments):
        chunk_starts.append(len(ftyp) + header + len(payload))
        for pos, size in ranges:
            payload += seg[pos:pos + size]
        base = len(durations)
        counts.append(len(ranges))
        durations += dur
        sync += [base + x for x in sy] if sy is not None else [base + i + 1 for i in range(len(ranges))]
        ctts += ct if ct is not None else [0] * len(ranges)
    total = sum(durations)
    mdat = struct.pack(">I4sQ", 1, b"mdat", header + len(payload)) + bytes(payload)
    sizes = [s for p in parsed for _, s in p[0]]
    stts = _full(b"stts", 0, 0, struct.pack(">I", len(_runs(durations)))
                 + b"".join(struct.pack(">II", c, d) for c, d in _runs(durations)))
    stsz = _full(b"stsz", 0, 0, struct.pack(">II", 0, len(sizes)) + struct.pack(f">{len(sizes)}I", *sizes))
    stsc = _full(b"stsc", 0, 0, struct.pack(">I", len(counts))
                 + b"".join(struct.pack(">III", i + 1, n, 1) for i, n in enumerate(counts)))
    co64 = _full(b"co64", 0, 0, struct.pack(">I", len(chunk_starts))
                 + struct.pack(f">{len(chunk_starts)}Q", *chunk_starts))
    stss = _full(b"stss", 0, 0, struct.pack(">I", len(sync)) + struct.pack(f">{len(sync)}I", *sync))
    new_ctts = b""
    if any(ctts):
        r = _runs(ctts)
        new_ctts = _full(b"ctts", 1, 0, struct.pack(">I", len(r))
                         + b"".join(struct.pack(">Ii", c, v) for c, v in r))
    tables = {b"stts": stts, b"stsz": stsz, b"stsc": stsc, b"stss": stss}

    def rebuild(off, size, movie_ts):
        """The box at off with its subtree rewritten for the joined video track."""
        kind = first[off + 4:off + 8]
        if kind == b"trak":
            mdia = _find_child(first, off, size, b"mdia")
            hdlr = _find_child(first, *mdia, b"hdlr")
            if first[hdlr[0] + 16:hdlr[0] + 20] != b"vide":
                raise ValueError("segments must be video-only")
        if kind in _CONTAINERS:
            parts = []
            for k, o, s in _children(first, off, size):
                if k == b"edts":
                    continue                        # the edit list described one segment
                if k == b"stbl":
                    sub = []
                    for kk, oo, ss in _children(first, o, s):
                        if kk in tables:
                            sub.append(tables[kk])
                        elif kk in (b"stco", b"co64"):
                            sub.append(co64)
                        elif kk == b"ctts":
                            sub.append(new_ctts)
                        else:
                            sub.append(first[oo:oo + ss])
                    if b"stss" not in {kk for kk, _, _ in _children(first, o, s)}:
                        sub.append(stss)
                    parts.append(_box(b"stbl", b"".join(sub)))
                else:
                    parts.append(rebuild(o, s, movie_ts))
            return _box(kind, b"".join(parts))
        raw = bytearray(first[off:off + size])
        v = raw[8]
        if kind == b"mvhd":
            at, fmt = (32, ">Q") if v == 1 else (24, ">I")
            raw[at:at + struct.calcsize(fmt)] = struct.pack(fmt, total * movie_ts // timescale)
        elif kind == b"tkhd":
            at, fmt = (36, ">Q") if v == 1 else (28, ">I")
            raw[at:at + struct.calcsize(fmt)] = struct.pack(fmt, total * movie_ts // timescale)
        elif kind == b"mdhd":
            at, fmt = (32, ">Q") if v == 1 else (24, ">I")
            raw[at:at + struct.calcsize(fmt)] = struct.pack(fmt, total)
        return bytes(raw)

    moov = next((o, s) for k, o, s in boxes(first) if k == b"moov")
    mvhd = _find_child(first, *moov, b"mvhd")
    at = mvhd[0] + (28 if first[mvhd[0] + 8] == 1 else 20)
    movie_ts = struct.unpack(">I", first[at:at + 4])[0]
    return ftyp + mdat + rebuild(*moov, movie_ts)
