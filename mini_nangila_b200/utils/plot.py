"""Line, point and bar charts as PNG or SVG with no plotting library.

matplotlib is not a dependency of this framework (and is absent on the
machines it targets), so the log plots of ``utils.analysis`` are drawn here:

    fig = Figure(width=900, height=400)
    ax = fig.add_axes(title="loss", xlabel="step", ylabel="loss")
    ax.line(x, y, color="tab:blue", label="train")
    ax.twin(ylabel="ratio").points(x2, r, color="tab:orange")
    fig.save("out.png")          # or "out.svg"

Each axes records its primitives in data coordinates; ``save`` lays out the
panels (stacked vertically), picks tick positions at 1/2/5 x 10^k steps and
emits either SVG elements or pixels: a numpy RGB canvas with lines stamped
as discs along each segment, alpha-blended points, filled bars and text in
an embedded 5x7 bitmap font (lower case shown in capitals), written as an
8-bit RGB PNG (zlib-deflated scanlines with filter 0, CRC-32 chunks).
"""
from __future__ import annotations

import math
import struct
import zlib

import numpy as np

COLORS = {
    "tab:blue": (31, 119, 180), "tab:orange": (255, 127, 14), "tab:green": (44, 160, 44),
    "tab:red": (214, 39, 40), "tab:purple": (148, 103, 189), "tab:brown": (140, 86, 75),
    "tab:pink": (227, 119, 194), "tab:gray": (127, 127, 127), "tab:olive": (188, 189, 34),
    "tab:cyan": (23, 190, 207), "black": (0, 0, 0), "gray": (128, 128, 128), "white": (255, 255, 255),
}
CYCLE = ["tab:blue", "tab:orange", "tab:green", "tab:red", "tab:purple", "tab:brown", "tab:pink", "tab:cyan"]

# 5x7 glyphs, one string per row, '#' = ink.
_GLYPHS = {
    " ": ".....|.....|.....|.....|.....|.....|.....",
    "0": ".###.|#...#|#..##|#.#.#|##..#|#...#|.###.", "1": "..#..|.##..|..#..|..#..|..#..|..#..|.###.",
    "2": ".###.|#...#|....#|...#.|..#..|.#...|#####", "3": "####.|....#|....#|.###.|....#|....#|####.",
    "4": "...#.|..##.|.#.#.|#..#.|#####|...#.|...#.", "5": "#####|#....|####.|....#|....#|#...#|.###.",
    "6": ".###.|#....|#....|####.|#...#|#...#|.###.", "7": "#####|....#|...#.|..#..|.#...|.#...|.#...",
    "8": ".###.|#...#|#...#|.###.|#...#|#...#|.###.", "9": ".###.|#...#|#...#|.####|....#|....#|.###.",
    "A": ".###.|#...#|#...#|#####|#...#|#...#|#...#", "B": "####.|#...#|#...#|####.|#...#|#...#|####.",
    "C": ".###.|#...#|#....|#....|#....|#...#|.###.", "D": "####.|#...#|#...#|#...#|#...#|#...#|####.",
    "E": "#####|#....|#....|####.|#....|#....|#####", "F": "#####|#....|#....|####.|#....|#....|#....",
    "G": ".###.|#...#|#....|#.###|#...#|#...#|.###.", "H": "#...#|#...#|#...#|#####|#...#|#...#|#...#",
    "I": ".###.|..#..|..#..|..#..|..#..|..#..|.###.", "J": "..###|...#.|...#.|...#.|...#.|#..#.|.##..",
    "K": "#...#|#..#.|#.#..|##...|#.#..|#..#.|#...#", "L": "#....|#....|#....|#....|#....|#....|#####",
    "M": "#...#|##.##|#.#.#|#.#.#|#...#|#...#|#...#", "N": "#...#|##..#|#.#.#|#..##|#...#|#...#|#...#",
    "O": ".###.|#...#|#...#|#...#|#...#|#...#|.###.", "P": "####.|#...#|#...#|####.|#....|#....|#....",
    "Q": ".###.|#...#|#...#|#...#|#.#.#|#..#.|.##.#", "R": "####.|#...#|#...#|####.|#.#..|#..#.|#...#",
    "S": ".####|#....|#....|.###.|....#|....#|####.", "T": "#####|..#..|..#..|..#..|..#..|..#..|..#..",
    "U": "#...#|#...#|#...#|#...#|#...#|#...#|.###.", "V": "#...#|#...#|#...#|#...#|#...#|.#.#.|..#..",
    "W": "#...#|#...#|#...#|#.#.#|#.#.#|#.#.#|.#.#.", "X": "#...#|#...#|.#.#.|..#..|.#.#.|#...#|#...#",
    "Y": "#...#|#...#|.#.#.|..#..|..#..|..#..|..#..", "Z": "#####|....#|...#.|..#..|.#...|#....|#####",
    ".": ".....|.....|.....|.....|.....|.##..|.##..", ",": ".....|.....|.....|.....|.##..|..#..|.#...",
    "-": ".....|.....|.....|.###.|.....|.....|.....", "+": ".....|..#..|..#..|#####|..#..|..#..|.....",
    "(": "...#.|..#..|.#...|.#...|.#...|..#..|...#.", ")": ".#...|..#..|...#.|...#.|...#.|..#..|.#...",
    "/": "....#|....#|...#.|..#..|.#...|#....|#....", "%": "##..#|##..#|...#.|..#..|.#...|#..##|#..##",
    "=": ".....|.....|#####|.....|#####|.....|.....", ":": ".....|.##..|.##..|.....|.##..|.##..|.....",
    "_": ".....|.....|.....|.....|.....|.....|#####", "[": ".###.|.#...|.#...|.#...|.#...|.#...|.###.",
    "]": ".###.|...#.|...#.|...#.|...#.|...#.|.###.", "'": "..#..|..#..|.#...|.....|.....|.....|.....",
    "<": "...#.|..#..|.#...|#....|.#...|..#..|...#.", ">": ".#...|..#..|...#.|....#|...#.|..#..|.#...",
    "!": "..#..|..#..|..#..|..#..|..#..|.....|..#..", "?": ".###.|#...#|....#|...#.|..#..|.....|..#..",
    "#": ".#.#.|.#.#.|#####|.#.#.|#####|.#.#.|.#.#.", "*": ".....|#.#.#|.###.|#####|.###.|#.#.#|.....",
    "^": "..#..|.#.#.|#...#|.....|.....|.....|.....", "|": "..#..|..#..|..#..|..#..|..#..|..#..|..#..",
    "~": ".....|.....|.#...|#.#.#|...#.|.....|.....", "&": ".##..|#..#.|#.#..|.#...|#.#.#|#..#.|.##.#",
}
_BITMAPS = {c: np.array([[ch == "#" for ch in row] for row in g.split("|")], dtype=bool) for c, g in _GLYPHS.items()}


def _rgb(color) -> tuple:
    if isinstance(color, tuple):
        return color
    if isinstance(color, str) and color.startswith("#") and len(color) == 7:
        return tuple(int(color[i:i + 2], 16) for i in (1, 3, 5))
    return COLORS.get(color, (0, 0, 0))


def nice_ticks(lo: float, hi: float, target: int = 6) -> list[float]:
    """Tick positions at 1, 2 or 5 x 10^k steps covering [lo, hi]."""
    if not (math.isfinite(lo) and math.isfinite(hi)):
        return [0.0]
    if hi <= lo:
        hi = lo + (abs(lo) if lo else 1.0)
    raw = (hi - lo) / max(1, target)
    mag = 10.0 ** math.floor(math.log10(raw))
    step = next(m * mag for m in (1, 2, 5, 10) if m * mag >= raw)
    first = math.ceil(lo / step - 1e-9) * step
    n = int(math.floor((hi - first) / step + 1e-9)) + 1
    return [first + i * step for i in range(max(1, n))]


def _fmt(v: float) -> str:
    if v == 0:
        return "0"
    if abs(v) >= 1e5 or abs(v) < 1e-3:
        return f"{v:.1e}"
    return f"{v:.4g}"


class Axes:
    """One panel: primitives in data coordinates, optional twin y axis."""

    def __init__(self, title: str = "", xlabel: str = "", ylabel: str = "", grid: bool = True):
        self.title, self.xlabel, self.ylabel, self.grid = title, xlabel, ylabel, grid
        self.items: list[tuple] = []
        self.xticklabels: list[str] | None = None
        self.secondary: Axes | None = None
        self._n = 0

    def _color(self, color):
        if color is None:
            color = CYCLE[self._n % len(CYCLE)]
            self._n += 1
        return _rgb(color)

    def line(self, x, y, color=None, label: str = "", width: float = 1.5, marker: bool = False):
        self.items.append(("line", np.asarray(x, float), np.asarray(y, float), self._color(color), label, width,
                           marker))
        return self

    def points(self, x, y, color=None, label: str = "", size: float = 2.5, alpha: float = 0.5):
        self.items.append(("points", np.asarray(x, float), np.asarray(y, float), self._color(color), label, size,
                           alpha))
        return self

    def bars(self, labels, heights, color=None, label: str = ""):
        h = np.asarray(heights, float)
        self.xticklabels = [str(s) for s in labels]
        self.items.append(("bars", np.arange(h.size, dtype=float), h, self._color(color), label, 0.7, None))
        return self

    def twin(self, ylabel: str = "") -> "Axes":
        self.secondary = Axes(ylabel=ylabel, grid=False)
        self.secondary._n = self._n
        return self.secondary

    def limits(self):
        xs = [i[1] for i in self.items] + ([i[1] for i in self.secondary.items] if self.secondary else [])
        ys = [i[2] for i in self.items]
        def rng(arrs, pad_zero=False):
            v = np.concatenate([a[np.isfinite(a)] for a in arrs]) if arrs else np.zeros(0)
            if v.size == 0:
                return 0.0, 1.0
            lo, hi = float(v.min()), float(v.max())
            if pad_zero:
                lo = min(lo, 0.0)
            if hi == lo:
                lo, hi = lo - 0.5, hi + 0.5
            return lo, hi
        has_bars = any(i[0] == "bars" for i in self.items)
        xl = rng(xs)
        if has_bars:
            xl = (xl[0] - 0.6, xl[1] + 0.6)
        return xl, rng(ys, pad_zero=has_bars)


class Figure:
    def __init__(self, width: int = 900, height: int = 420):
        self.width, self.height = int(width), int(height)
        self.axes: list[Axes] = []

    def add_axes(self, **kw) -> Axes:
        ax = Axes(**kw)
        self.axes.append(ax)
        return ax

    # ---------------------------------------------------------------- layout
    def _panels(self):
        n = max(1, len(self.axes))
        ph = self.height / n
        out = []
        for i, ax in enumerate(self.axes):
            left, right = 80, self.width - (80 if ax.secondary else 30)
            top, bottom = i * ph + (30 if ax.title else 15), (i + 1) * ph - (70 if ax.xticklabels else 50)
            out.append((ax, left, right, top, bottom))
        return out

    def _scene(self):
        """Device-independent drawing list: ('line', pts, rgb, width), ('rect', x0, y0, x1, y1, rgb),
        ('dot', x, y, r, rgb, alpha), ('text', x, y, s, rgb, anchor, vertical)."""
        ops = [("rect", 0, 0, self.width, self.height, (255, 255, 255))]
        for ax, L, R, T, B in self._panels():
            (x0, x1), (y0, y1) = ax.limits()
            xt, yt = nice_ticks(x0, x1), nice_ticks(y0, y1)
            x0, x1 = min(x0, xt[0]), max(x1, xt[-1])
            y0, y1 = min(y0, yt[0]), max(y1, yt[-1])
            fx = lambda v, x0=x0, x1=x1, L=L, R=R: L + (v - x0) / (x1 - x0) * (R - L)
            fy = lambda v, y0=y0, y1=y1, T=T, B=B: B - (v - y0) / (y1 - y0) * (B - T)
            if ax.grid:
                for t in yt:
                    ops.append(("line", [(L, fy(t)), (R, fy(t))], (225, 225, 225), 1.0))
            if ax.xticklabels is None:
                for t in xt:
                    ops.append(("line", [(fx(t), B), (fx(t), B + 4)], (0, 0, 0), 1.0))
                    ops.append(("text", fx(t), B + 8, _fmt(t), (0, 0, 0), "top", False))
            else:
                for i, s in enumerate(ax.xticklabels):
                    ops.append(("text", fx(i), B + 8, s, (0, 0, 0), "top", False))
            for t in yt:
                ops.append(("line", [(L - 4, fy(t)), (L, fy(t))], (0, 0, 0), 1.0))
                ops.append(("text", L - 7, fy(t), _fmt(t), (0, 0, 0), "right", False))
            legend = []
            for it in ax.items:
                ops += self._item_ops(it, fx, fy, B)
                if it[4]:
                    legend.append((it[4], it[3]))
            if ax.secondary is not None and ax.secondary.items:
                sx = ax.secondary
                _, (s0, s1) = sx.limits()
                st = nice_ticks(s0, s1)
                s0, s1 = min(s0, st[0]), max(s1, st[-1])
                gy = lambda v, s0=s0, s1=s1, T=T, B=B: B - (v - s0) / (s1 - s0) * (B - T)
                for it in sx.items:
                    ops += self._item_ops(it, fx, gy, B)
                    if it[4]:
                        legend.append((it[4], it[3]))
                for t in st:
                    ops.append(("line", [(R, gy(t)), (R + 4, gy(t))], (0, 0, 0), 1.0))
                    ops.append(("text", R + 7, gy(t), _fmt(t), (0, 0, 0), "left", False))
                if sx.ylabel:
                    ops.append(("text", self.width - 12, (T + B) / 2, sx.ylabel, (0, 0, 0), "center", True))
            ops.append(("line", [(L, T), (R, T), (R, B), (L, B), (L, T)], (0, 0, 0), 1.0))
            if ax.title:
                ops.append(("text", (L + R) / 2, T - 18, ax.title, (0, 0, 0), "center", False))
            if ax.xlabel:
                ops.append(("text", (L + R) / 2, B + (44 if ax.xticklabels else 26), ax.xlabel, (0, 0, 0), "center",
                            False))
            if ax.ylabel:
                ops.append(("text", 14, (T + B) / 2, ax.ylabel, (0, 0, 0), "center", True))
            for k, (lab, rgb) in enumerate(legend):
                y = T + 12 + 14 * k
                ops.append(("line", [(R - 150, y), (R - 130, y)], rgb, 2.0))
                ops.append(("text", R - 125, y, lab, (0, 0, 0), "left", False))
        return ops

    @staticmethod
    def _item_ops(it, fx, fy, B):
        kind, x, y, rgb, _, a, b = it
        ok = np.isfinite(x) & np.isfinite(y)
        x, y = x[ok], y[ok]
        if kind == "line":
            out = [("line", [(fx(u), fy(v)) for u, v in zip(x, y)], rgb, a)] if x.size > 1 else []
            if b or x.size == 1:
                out += [("dot", fx(u), fy(v), 2.5, rgb, 1.0) for u, v in zip(x, y)]
            return out
        if kind == "points":
            return [("dot", fx(u), fy(v), a, rgb, b) for u, v in zip(x, y)]
        half = a / 2
        return [("rect", fx(u - half), fy(max(v, 0.0)), fx(u + half), fy(min(v, 0.0)), rgb) for u, v in zip(x, y)]

    # ------------------------------------------------------------ back ends
    def to_svg(self) -> str:
        def col(c):
            return "rgb(%d,%d,%d)" % c

        def esc(s):
            return s.replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")

        parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{self.width}" height="{self.height}" '
                 f'font-family="sans-serif" font-size="11">']
        for op in self._scene():
            if op[0] == "rect":
                _, x0, y0, x1, y1, c = op
                parts.append(f'<rect x="{min(x0, x1):.1f}" y="{min(y0, y1):.1f}" width="{abs(x1 - x0):.1f}" '
                             f'height="{abs(y1 - y0):.1f}" fill="{col(c)}"/>')
            elif op[0] == "line":
                pts = " ".join(f"{x:.1f},{y:.1f}" for x, y in op[1])
                parts.append(f'<polyline points="{pts}" fill="none" stroke="{col(op[2])}" stroke-width="{op[3]}"/>')
            elif op[0] == "dot":
                _, x, y, r, c, a = op
                parts.append(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="{r}" fill="{col(c)}" fill-opacity="{a}"/>')
            else:
                _, x, y, s, c, anchor, vert = op
                ta = {"right": "end", "left": "start"}.get(anchor, "middle")
                base = "hanging" if anchor == "top" else "middle"
                rot = f' transform="rotate(-90 {x:.1f} {y:.1f})"' if vert else ""
                parts.append(f'<text x="{x:.1f}" y="{y:.1f}" text-anchor="{ta}" dominant-baseline="{base}" '
                             f'fill="{col(c)}"{rot}>{esc(s)}</text>')
        parts.append("</svg>")
        return "\n".join(parts)

    def to_pixels(self) -> np.ndarray:
        img = np.full((self.height, self.width, 3), 255, dtype=np.uint8)
        for op in self._scene():
            if op[0] == "rect":
                _, x0, y0, x1, y1, c = op
                xa, xb = sorted((int(round(x0)), int(round(x1))))
                ya, yb = sorted((int(round(y0)), int(round(y1))))
                img[max(0, ya):max(0, yb), max(0, xa):max(0, xb)] = c
            elif op[0] == "line":
                _stroke(img, op[1], op[2], op[3])
            elif op[0] == "dot":
                _, x, y, r, c, a = op
                _disc(img, x, y, r, c, a)
            else:
                _, x, y, s, c, anchor, vert = op
                _text(img, x, y, s, c, anchor, vert)
        return img

    def to_png(self) -> bytes:
        return png_bytes(self.to_pixels())

    def save(self, path: str) -> str:
        data = self.to_svg().encode() if path.lower().endswith(".svg") else self.to_png()
        with open(path, "wb") as fh:
            fh.write(data)
        return path


# ------------------------------------------------------------- rasterising
def _disc(img, x, y, r, c, alpha=1.0):
    h, w, _ = img.shape
    x0, x1 = int(math.floor(x - r)), int(math.ceil(x + r)) + 1
    y0, y1 = int(math.floor(y - r)), int(math.ceil(y + r)) + 1
    xa, xb, ya, yb = max(0, x0), min(w, x1), max(0, y0), min(h, y1)
    if xa >= xb or ya >= yb:
        return
    yy, xx = np.mgrid[ya:yb, xa:xb]
    m = (xx + 0.5 - x) ** 2 + (yy + 0.5 - y) ** 2 <= r * r + 0.25
    sub = img[ya:yb, xa:xb]
    sub[m] = (sub[m] * (1 - alpha) + np.asarray(c) * alpha).astype(np.uint8)


def _stroke(img, pts, c, width):
    h, w, _ = img.shape
    r = max(0.5, width / 2)
    samples = []
    for (xa, ya), (xb, yb) in zip(pts[:-1], pts[1:]):
        n = max(2, int(math.hypot(xb - xa, yb - ya) * 2) + 1)
        t = np.linspace(0.0, 1.0, n)
        samples.append(np.stack([xa + (xb - xa) * t, ya + (yb - ya) * t], 1))
    if not samples:
        return
    s = np.concatenate(samples)
    ri = int(math.ceil(r))
    for dy in range(-ri, ri + 1):
        for dx in range(-ri, ri + 1):
            if dx * dx + dy * dy > r * r + 0.25:
                continue
            px = np.round(s[:, 0] + dx).astype(np.int64)
            py = np.round(s[:, 1] + dy).astype(np.int64)
            ok = (px >= 0) & (px < w) & (py >= 0) & (py < h)
            img[py[ok], px[ok]] = c


def _text(img, x, y, s, c, anchor="left", vertical=False, scale=2):
    s = s.upper()
    gw, gh, adv = 5 * scale, 7 * scale, 6 * scale
    n = len(s)
    tw = n * adv - scale
    glyphs = np.zeros((gh, max(1, tw)), dtype=bool)
    for i, ch in enumerate(s):
        g = _BITMAPS.get(ch, _BITMAPS["?"] if ch != " " else _BITMAPS[" "])
        glyphs[:, i * adv:i * adv + gw] |= np.kron(g, np.ones((scale, scale), dtype=bool))
    if vertical:
        glyphs = np.rot90(glyphs)
    bh, bw = glyphs.shape
    if vertical:
        x0, y0 = x - bw / 2, y - bh / 2
    elif anchor == "right":
        x0, y0 = x - bw, y - bh / 2
    elif anchor == "left":
        x0, y0 = x, y - bh / 2
    elif anchor == "top":
        x0, y0 = x - bw / 2, y
    else:
        x0, y0 = x - bw / 2, y - bh / 2
    x0, y0 = int(round(x0)), int(round(y0))
    h, w, _ = img.shape
    ya, yb, xa, xb = max(0, y0), min(h, y0 + bh), max(0, x0), min(w, x0 + bw)
    if ya >= yb or xa >= xb:
        return
    m = glyphs[ya - y0:yb - y0, xa - x0:xb - x0]
    img[ya:yb, xa:xb][m] = c


def png_bytes(img: np.ndarray) -> bytes:
    """8-bit RGB PNG of an (H, W, 3) uint8 array."""
    img = np.ascontiguousarray(img, dtype=np.uint8)
    h, w, _ = img.shape
    raw = b"".join(b"\x00" + img[r].tobytes() for r in range(h))

    def chunk(tag: bytes, data: bytes) -> bytes:
        return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)

    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0))
            + chunk(b"IDAT", zlib.compress(raw, 6)) + chunk(b"IEND", b""))


def read_png(data: bytes) -> np.ndarray:
    """Decode an 8-bit RGB, non-interlaced PNG with filter 0 rows (what
    ``png_bytes`` writes) back to an array; for tests."""
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    p, idat, w, h = 8, b"", 0, 0
    while p < len(data):
        n = struct.unpack(">I", data[p:p + 4])[0]
        tag, body = data[p + 4:p + 8], data[p + 8:p + 8 + n]
        assert struct.unpack(">I", data[p + 8 + n:p + 12 + n])[0] == zlib.crc32(tag + body) & 0xFFFFFFFF
        if tag == b"IHDR":
            w, h = struct.unpack(">II", body[:8])
        elif tag == b"IDAT":
            idat += body
        p += 12 + n
    raw = zlib.decompress(idat)
    rows = [raw[r * (3 * w + 1) + 1:(r + 1) * (3 * w + 1)] for r in range(h)]
    return np.frombuffer(b"".join(rows), dtype=np.uint8).reshape(h, w, 3)
