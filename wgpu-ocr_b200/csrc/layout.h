// Host half of the ocrs page pipeline (src/bin/ocr-bench.rs:458-585 without DET / REC): word
// rectangles grouped into text lines (ocrs' find_text_lines, src/bin/ocr-bench.rs:516), the lines
// padded (src/bin/ocr-bench.rs:534-558) and each line's crop and polygon for the device line
// images (ocrs' prepare_recognition_input, src/bin/ocr-bench.rs:365-408).  ocrs =0.13.1 is not
// vendored: its rules are restated from its documented behaviour (layout.cpp states them).
#pragma once

#include <cstdint>
#include <vector>

namespace wocr {

// Rotated rectangles are [cx, cy, up_x, up_y, width, height], as word_rects writes them.
constexpr int kLineHeight = 64;      // ocrs recognition input height
constexpr int kLineMinWidth = 10, kLineMaxWidth = 800;
constexpr int kLineBucket = 50, kLinesPerBatch = 20;  // line_batches grouping
constexpr int kMaxLineVerts = 2048;  // 512 words a line

// The words of each text line: `order` lists word indices line by line (each left to right),
// `line_len` the words of each line; lines in reading order.
void text_lines(const float *words, int n, std::vector<int> &order, std::vector<int> &line_len);

// One line's words (in place): relv x the median word height across the text on both sides,
// relend x it along the text at the line's two ends.
void pad_line(float *words, int nw, float relv, float relend);

// A line's crop on a pw x ph page and its image width; its polygon's vertices (x, y pairs) are
// appended to `vxy`.
struct LineCut {
    int l = 0, t = 0, cw = 1, ch = 1, W = kLineMinWidth;
};
LineCut line_cut(const float *words, int nw, int pw, int ph, std::vector<int> &vxy);

}  // namespace wocr
