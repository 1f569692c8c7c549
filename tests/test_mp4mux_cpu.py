"""The MP4 muxer: the PCM track added to OpenCV's video-only mp4 points at exactly the
samples given (chunk offset, sample count, sample size, rate), the movie header's next
track id and duration are updated, and the video track still decodes."""
import struct

import numpy as np
import pytest

from vdn_minimax_h3_b200.inference.mp4mux import add_pcm_track, boxes, track_handlers


def _find(data, path, start=0, end=None):
    """Offset and size of the first box along a path of box types."""
    for kind in path:
        hit = next(((o, s) for k, o, s in boxes(data, start, end) if k == kind), None)
        if hit is None:
            return None
        start, end = hit[0] + 8, hit[0] + hit[1]
    return hit


def test_pcm_track_round_trip(tmp_path):
    cv2 = pytest.importorskip("cv2")
    path = str(tmp_path / "v.mp4")
    w = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), 24, (64, 48))
    for i in range(10):
        w.write(np.full((48, 64, 3), 20 * i, np.uint8))
    w.release()
    video = open(path, "rb").read()
    rng = np.random.default_rng(0)
    pcm = rng.integers(-30000, 30000, size=(20000, 2), dtype=np.int16)
    out = add_pcm_track(video, pcm, 48000)
    assert out[:len(video) - (len(video) - [o for k, o, s in boxes(video) if k == b"moov"][0])] == \
        video[:[o for k, o, s in boxes(video) if k == b"moov"][0]]
    assert track_handlers(out) == [b"vide", b"soun"]
    moov = _find(out, [b"moov"])
    traks = [(o, s) for k, o, s in boxes(out, moov[0] + 8, moov[0] + moov[1]) if k == b"trak"]
    o, s = traks[1]
    stbl = _find(out, [b"mdia", b"minf", b"stbl"], o + 8, o + s)
    so, ss = _find(out, [b"stco"], stbl[0] + 8, stbl[0] + stbl[1])
    count, offset = struct.unpack(">II", out[so + 12:so + 20])
    zo, zs = _find(out, [b"stsz"], stbl[0] + 8, stbl[0] + stbl[1])
    size, n = struct.unpack(">II", out[zo + 12:zo + 20])
    assert count == 1 and size == 4 and n == 20000
    assert np.array_equal(np.frombuffer(out[offset:offset + 4 * n], dtype="<i2").reshape(-1, 2), pcm)
    mdhd = _find(out, [b"mdia", b"mdhd"], o + 8, o + s)
    rate, dur = struct.unpack(">II", out[mdhd[0] + 20:mdhd[0] + 28])
    assert (rate, dur) == (48000, 20000)
    mvhd = _find(out, [b"moov", b"mvhd"])
    assert struct.unpack(">I", out[mvhd[0] + mvhd[1] - 4:mvhd[0] + mvhd[1]])[0] == 3
    open(path, "wb").write(out)
    cap = cv2.VideoCapture(path)
    frames = 0
    while cap.read()[0]:
        frames += 1
    assert frames == 10


def test_refuses_moov_first():
    with pytest.raises(ValueError):
        add_pcm_track(struct.pack(">I4s", 8, b"moov") + struct.pack(">I4s", 8, b"mdat"),
                      np.zeros((4, 2), np.int16), 48000)


def test_concat_segments_decodes_like_its_parts(tmp_path):
    """Segments encoded separately and joined into one track decode, frame for frame, to
    exactly what each segment decodes to on its own (the samples are copied verbatim), with
    one sync sample per segment start at least, and the soundtrack can still be muxed."""
    cv2 = pytest.importorskip("cv2")
    from vdn_minimax_h3_b200.inference.mp4mux import concat_video_segments

    def frame(i):
        y, x = np.mgrid[0:48, 0:64]
        return np.stack([(x * 4 + i * 7) % 256, (y * 5 + i * 3) % 256,
                         np.full_like(x, 10 * i % 256)], -1).astype(np.uint8)

    def encode(idx, path):
        w = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), 24, (64, 48))
        for i in idx:
            w.write(frame(i))
        w.release()
        return open(path, "rb").read()

    def decode(path):
        cap, out = cv2.VideoCapture(path), []
        while True:
            ok, f = cap.read()
            if not ok:
                return out
            out.append(f)

    parts = [range(0, 9), range(9, 20), range(20, 30)]
    segs = [encode(r, str(tmp_path / f"s{i}.mp4")) for i, r in enumerate(parts)]
    joined = concat_video_segments(segs)
    path = str(tmp_path / "joined.mp4")
    open(path, "wb").write(joined)
    got = decode(path)
    want = [f for i in range(3) for f in decode(str(tmp_path / f"s{i}.mp4"))]
    assert len(got) == 30 and all(np.array_equal(a, b) for a, b in zip(got, want))
    muxed = add_pcm_track(joined, np.zeros((4800, 2), np.int16), 48000)
    assert track_handlers(muxed) == [b"vide", b"soun"]
    open(path, "wb").write(muxed)
    assert len(decode(path)) == 30


def test_concat_many_small_segments(tmp_path):
    """The split encode of 8 ranks x several writers hands the join up to ~40 segments, some
    of a single frame: all of them join into one track that decodes like its parts."""
    cv2 = pytest.importorskip("cv2")
    from vdn_minimax_h3_b200.inference.mp4mux import concat_video_segments
    from vdn_minimax_h3_b200.inference.vae import encode_mp4

    rng = np.random.default_rng(0)
    frames = rng.integers(0, 255, size=(61, 32, 48, 3), dtype=np.uint8)
    frames[:, :16] = 40                                   # some structure for the codec
    cuts = [0, 1, 3, 4, 8, 9, 15, 16, 17, 25, 26, 27, 40, 41, 55, 60, 61]
    segs = []
    for i in range(len(cuts) - 1):
        path = str(tmp_path / f"s{i}.mp4")
        w = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), 24, (48, 32))
        for f in frames[cuts[i]:cuts[i + 1]]:
            w.write(np.ascontiguousarray(f[:, :, ::-1]))
        w.release()
        segs.append(open(path, "rb").read())
    joined = str(tmp_path / "joined.mp4")
    open(joined, "wb").write(concat_video_segments(segs))

    def decode(path):
        cap, out = cv2.VideoCapture(path), []
        while True:
            ok, f = cap.read()
            if not ok:
                return out
            out.append(f)

    got = decode(joined)
    want = [f for i in range(len(segs)) for f in decode(str(tmp_path / f"s{i}.mp4"))]
    assert len(got) == 61 and all(np.array_equal(a, b) for a, b in zip(got, want))
    # and the encoder's own split (ranges of >= 8 frames on several writers) gives every frame
    import torch
    data = encode_mp4(torch.from_numpy(frames), workers=6)
    path = str(tmp_path / "split.mp4")
    open(path, "wb").write(data)
    assert len(decode(path)) == 61
