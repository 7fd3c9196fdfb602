"""The host half of the ocrs page pipeline in the library (`wocr_text_lines`, `wocr_pad_line`)
against the oracle's restatement of ocrs' line grouping and the reference's line padding
(src/bin/ocr-bench.rs:516, 534-558).  Host code only: no device is needed."""
import numpy as np
import pytest

import wocr
from oracle import ref
from wocr import synth


def _random_words(seed, n, rotate=False):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        cx, cy = rng.uniform(0, 1200), rng.uniform(0, 900)
        w, h = rng.uniform(8, 120), rng.uniform(8, 40)
        if rotate:
            a = rng.uniform(-0.3, 0.3)
            up = (np.sin(a), -np.cos(a))
            if rng.random() < 0.2:              # up axis nearer horizontal: width and height swap
                up = (-np.cos(a), -np.sin(a))
                w, h = h, w
            if rng.random() < 0.3:              # up pointing down
                up = (-up[0], -up[1])
        else:
            up = (0.0, -1.0) if rng.random() < 0.5 else (0.0, 1.0)
        out.append([cx, cy, up[0], up[1], w, h])
    return np.array(out, np.float32).reshape(-1, 6)


def _page_words(seed):
    bits = synth.pack_mask(synth.page_word_mask(seed, 1275, 1650, bands=18, line_h=20, grow_x=4, grow_y=2))
    return ref.word_rects(bits, 1275, 1650)


@pytest.mark.parametrize("case", ["page0", "page1", "random", "rotated", "banded", "one", "none"])
def test_text_lines_equal_oracle(case):
    if case.startswith("page"):
        words = _page_words(int(case[-1]) + 11)
    elif case == "random":
        words = _random_words(1, 300)
    elif case == "rotated":
        words = _random_words(2, 200, rotate=True)
    elif case == "banded":            # rows of words at the 5 px overlap and gap limits
        rows = []
        for r in range(6):
            x = 10.0
            for k in range(12):
                w = 20.0 + 3 * k
                rows.append([x + w / 2, 40.0 + r * 30.0 + (k % 3) * 2.5, 0.0, -1.0, w, 12.0])
                x += w - 5.0 + (k % 4) * 2.5         # some at -5 px (allowed), some beyond
        words = np.array(rows, np.float32)
    elif case == "one":
        words = _random_words(3, 1)
    else:
        words = np.zeros((0, 6), np.float32)
    got = wocr.text_lines(words)
    want = ref.text_lines(words)
    assert got == want
    flat = sorted(i for line in got for i in line)
    assert flat == list(range(len(words)))          # every word in exactly one line
    if case.startswith("page"):
        assert 10 <= len(got) <= 18 * 2


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_pad_line_equal_oracle(seed):
    words = _random_words(seed + 20, 9, rotate=True)
    for k in (1, 2, 9):
        np.testing.assert_array_equal(wocr.pad_line(words[:k]), ref.pad_line(words[:k]))
        np.testing.assert_array_equal(wocr.pad_line(words[:k], 0.3, 0.0), ref.pad_line(words[:k], 0.3, 0.0))


def test_pad_line_rule():
    """src/bin/ocr-bench.rs:534-558 on an upright line: the median height (sorted, element n / 2),
    0.15 of it above and below every word, 0.1 of it at the two ends."""
    words = np.array([[10, 10, 0, -1, 10, 20], [30, 10, 0, -1, 10, 30], [50, 10, 0, -1, 10, 40]], np.float32)
    p = wocr.pad_line(words)
    med = np.float32(30)
    np.testing.assert_array_equal(p[:, 5], words[:, 5] + np.float32(2) * (np.float32(0.15) * med))
    np.testing.assert_array_equal(p[:, 4], words[:, 4] + np.float32(2) * np.array([np.float32(0.1) * med, 0,
                                                                                    np.float32(0.1) * med], np.float32))
