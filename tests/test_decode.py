"""The host-side greedy CTC decoders and the PP-OCR dictionary loader against the reference's
rules, with known answers worked out from them (src/bin/ocr-bench.rs:62-74 for ocrs,
src/ppocr.rs:10-33 for PP-OCR).  CPU only."""
import wocr
from wocr import synth


def test_pp_decode_rules():
    """Blanks dropped, repeats merged (a blank between repeats keeps both), classes past the
    dictionary give nothing."""
    chars = ["", "a", "b", " "]
    assert wocr.pp_decode([0, 1, 1, 0, 1, 2, 2, 3, 0, 3], chars) == "aab  "
    assert wocr.pp_decode([], chars) == ""
    assert wocr.pp_decode([0, 0, 0], chars) == ""
    assert wocr.pp_decode([2, 9, 9, 2], chars) == "bb"          # class 9 is past the list


def test_ocrs_decode_rules():
    """Class c is ALPHABET[c - 1]; blanks dropped, repeats merged, steps t with t * 4 >= width
    (the line's padding) dropped, and only `steps` steps read."""
    a = synth.OCRS_ALPHABET
    best = [0, 12, 12, 0, 12, 13, 13, 14, 14, 15]
    assert wocr.ocrs_decode(best, 10, 40, a) == a[11] + a[11] + a[12] + a[13] + a[14]
    assert wocr.ocrs_decode(best, 10, 24, a) == a[11] + a[11] + a[12]   # t = 6.. are padding
    assert wocr.ocrs_decode(best, 3, 40, a) == a[11]
    assert wocr.ocrs_decode([1, 1, 2], 3, 12, a) == " " + "0"


def test_load_pp_dictionary(tmp_path):
    """Blank first, the lines in order (CRLF and a final newline as Rust's str::lines reads
    them), the space last."""
    p = tmp_path / "dict.txt"
    p.write_bytes("x\r\ny\n\nz\n".encode())
    assert wocr.load_pp_dictionary(str(p)) == ["", "x", "y", "", "z", " "]
    p.write_bytes("x\ny".encode())
    assert wocr.load_pp_dictionary(str(p)) == ["", "x", "y", " "]
