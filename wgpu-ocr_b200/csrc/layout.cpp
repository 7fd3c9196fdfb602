// Host half of the ocrs page pipeline: text lines, line padding, line crops and polygons.
//
// ocrs =0.13.1 (find_text_lines and prepare_recognition_input, called by the reference at
// src/bin/ocr-bench.rs:516 and 365-408) is an un-vendored crates.io dependency, so these rules are
// a restatement of its documented behaviour (parity against ocrs itself is unpinned):
//
// * Lines: words by the integer part of their bounding rectangle's left edge (stable).  A line
//   begins with the first word not yet placed and takes, again and again, the unplaced word
//   with the smallest left edge among those starting no more than 5 px left of the line's last
//   word's right edge and overlapping it vertically by 5 px or more.  Lines are then ordered by
//   the top edge of their first word (stable).  ocrs's column separators (from empty page
//   regions) are not restated: the single-column synthetic pages have none.
// * Padding (src/bin/ocr-bench.rs:534-558): the median of the words' heights (the side across
//   the text: height when the up axis is nearer vertical, else width); every word grows by
//   relv x median across the text on both sides, the first and last by relend x median along it.
// * Line polygon: per word, left to right, the two corners of its top edge, then per word, right
//   to left, the two corners of its bottom edge, truncated to integers (Rust `as i32`).  A word's
//   top edge lies along the one of up, -up, right = (-up.y, up.x), -right that points most
//   upward (smallest y; the first on ties).  The crop is the polygon's bounding rectangle
//   clamped to the page (at least 1 x 1) and the image is 64 x W, W = (int) clamp(64 cw / ch,
//   10, 800).
#include "layout.h"

#include <algorithm>
#include <cmath>
#include <numeric>

namespace wocr {

namespace {

struct Box {
    float l, t, r, b;
};

// bounding rectangle of a rotated rect from its four corners
Box bounds(const float *w) {
    const float hw = w[4] / 2.0f, hh = w[5] / 2.0f;
    Box b{INFINITY, INFINITY, -INFINITY, -INFINITY};
    for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
            const float along = (float)sa * hh, across = (float)sb * hw;
            const float x = w[0] + along * w[2] + across * -w[3];
            const float y = w[1] + along * w[3] + across * w[2];
            b.l = std::min(b.l, x);
            b.r = std::max(b.r, x);
            b.t = std::min(b.t, y);
            b.b = std::max(b.b, y);
        }
    return b;
}

bool upright(const float *w) { return std::fabs(w[3]) >= std::fabs(w[2]); }

}  // namespace

void text_lines(const float *words, int n, std::vector<int> &order, std::vector<int> &line_len) {
    order.clear();
    line_len.clear();
    if (n <= 0) return;
    std::vector<Box> bx((size_t)n);
    for (int i = 0; i < n; i++) bx[i] = bounds(words + 6 * (size_t)i);
    std::vector<int> sorted((size_t)n);
    std::iota(sorted.begin(), sorted.end(), 0);
    std::stable_sort(sorted.begin(), sorted.end(), [&](int a, int b) { return (int)bx[a].l < (int)bx[b].l; });
    std::vector<char> placed((size_t)n, 0);
    std::vector<std::vector<int>> lines;
    for (int start : sorted) {
        if (placed[start]) continue;
        std::vector<int> line{start};
        placed[start] = 1;
        while (true) {
            const Box &last = bx[line.back()];
            int pick = -1;
            for (int c : sorted) {
                if (placed[c]) continue;
                const Box &cb = bx[c];
                const float overlap = std::min(last.b, cb.b) - std::max(last.t, cb.t);
                if (!(cb.l >= last.r - 5.0f) || !(overlap >= 5.0f)) continue;
                if (pick < 0 || cb.l < bx[pick].l) pick = c;
            }
            if (pick < 0) break;
            placed[pick] = 1;
            line.push_back(pick);
        }
        lines.push_back(std::move(line));
    }
    std::stable_sort(lines.begin(), lines.end(),
                     [&](const std::vector<int> &a, const std::vector<int> &b) { return bx[a[0]].t < bx[b[0]].t; });
    for (const auto &l : lines) {
        line_len.push_back((int)l.size());
        order.insert(order.end(), l.begin(), l.end());
    }
}

void pad_line(float *words, int nw, float relv, float relend) {
    if (nw <= 0) return;
    std::vector<float> hs((size_t)nw);
    for (int i = 0; i < nw; i++) {
        const float *w = words + 6 * (size_t)i;
        hs[i] = upright(w) ? w[5] : w[4];
    }
    std::sort(hs.begin(), hs.end());
    const float med = hs[(size_t)nw / 2];
    for (int i = 0; i < nw; i++) {
        float *w = words + 6 * (size_t)i;
        const float along = (i == 0 || i == nw - 1) ? relend * med : 0.0f;
        const float across = relv * med;
        const float grow_w = upright(w) ? along : across, grow_h = upright(w) ? across : along;
        w[4] = w[4] + 2.0f * grow_w;
        w[5] = w[5] + 2.0f * grow_h;
    }
}

LineCut line_cut(const float *words, int nw, int pw, int ph, std::vector<int> &vxy) {
    LineCut lc;
    if (nw <= 0) return lc;
    const size_t v0 = vxy.size();
    vxy.resize(v0 + (size_t)8 * nw);
    int *v = vxy.data() + v0;
    for (int i = 0; i < nw; i++) {
        const float *w = words + 6 * (size_t)i;
        const float hw = w[4] / 2.0f, hh = w[5] / 2.0f;
        // the most upward of up, -up, right, -right, with its half extent and the other one
        float ux = w[2], uy = w[3], eu = hh, er = hw;
        const float cand[3][3] = {{-w[2], -w[3], hh}, {-w[3], w[2], hw}, {w[3], -w[2], hw}};
        for (int q = 0; q < 3; q++)
            if (cand[q][1] < uy) {
                ux = cand[q][0];
                uy = cand[q][1];
                eu = cand[q][2];
                er = q == 0 ? hw : hh;
            }
        const float rx = -uy, ry = ux;
        const float tx = w[0] + eu * ux, ty = w[1] + eu * uy;
        const float bx_ = w[0] - eu * ux, by_ = w[1] - eu * uy;
        int *top = v + 4 * i;                        // top-left, top-right
        int *bot = v + 4 * (2 * nw - 1 - i);         // bottom-right, bottom-left
        top[0] = (int)(tx - er * rx);
        top[1] = (int)(ty - er * ry);
        top[2] = (int)(tx + er * rx);
        top[3] = (int)(ty + er * ry);
        bot[0] = (int)(bx_ + er * rx);
        bot[1] = (int)(by_ + er * ry);
        bot[2] = (int)(bx_ - er * rx);
        bot[3] = (int)(by_ - er * ry);
    }
    int mnx = v[0], mxx = v[0], mny = v[1], mxy = v[1];
    for (int k = 1; k < 4 * nw; k++) {
        mnx = std::min(mnx, v[2 * k]);
        mxx = std::max(mxx, v[2 * k]);
        mny = std::min(mny, v[2 * k + 1]);
        mxy = std::max(mxy, v[2 * k + 1]);
    }
    lc.l = std::clamp(mnx, 0, pw - 1);
    lc.t = std::clamp(mny, 0, ph - 1);
    const int r = std::clamp(mxx, lc.l + 1, pw), b = std::clamp(mxy, lc.t + 1, ph);
    lc.cw = r - lc.l;
    lc.ch = b - lc.t;
    const float fw = (float)kLineHeight * (float)lc.cw / (float)lc.ch;
    lc.W = (int)std::min(std::max(fw, (float)kLineMinWidth), (float)kLineMaxWidth);
    return lc;
}

}  // namespace wocr
