"""A minimal RGB canvas written as PNG (zlib + CRC chunks, no plotting
library). Used for the pipeline Gantt charts; draws filled rectangles, lines
and text in a built-in 5x7 bitmap font (upper-case letters, digits and a few
symbols)."""

from __future__ import annotations

import struct
import zlib
from typing import Tuple

Color = Tuple[int, int, int]

# 5x7 glyphs, one string of 7 rows x 5 columns per character ('#' = set).
_FONT = {
    "0": "01110100011001110101110011000101110", "1": "00100011000010000100001000010001110",
    "2": "01110100010000100010001000100011111", "3": "11111000100010000010000011000101110",
    "4": "00010001100101010010111110001000010", "5": "11111100001111000001000011000101110",
    "6": "00110010001000011110100011000101110", "7": "11111000010001000100010000100001000",
    "8": "01110100011000101110100011000101110", "9": "01110100011000101111000010001001100",
    "A": "01110100011000111111100011000110001", "B": "11110100011000111110100011000111110",
    "C": "01110100011000010000100001000101110", "D": "11100100101000110001100011001011100",
    "E": "11111100001000011110100001000011111", "F": "11111100001000011110100001000010000",
    "G": "01110100011000010111100011000101111", "H": "10001100011000111111100011000110001",
    "I": "01110001000010000100001000010001110", "J": "00111000100001000010000101001001100",
    "K": "10001100101010011000101001001010001", "L": "10000100001000010000100001000011111",
    "M": "10001110111010110101100011000110001", "N": "10001100011100110101100111000110001",
    "O": "01110100011000110001100011000101110", "P": "11110100011000111110100001000010000",
    "Q": "01110100011000110001101011001001101", "R": "11110100011000111110101001001010001",
    "S": "01111100001000001110000010000111110", "T": "11111001000010000100001000010000100",
    "U": "10001100011000110001100011000101110", "V": "10001100011000110001100010101000100",
    "W": "10001100011000110101101011010101010", "X": "10001100010101000100010101000110001",
    "Y": "10001100011000101010001000010000100", "Z": "11111000010001000100010001000011111",
    " ": "00000000000000000000000000000000000", ".": "00000000000000000000000000110001100",
    ":": "00000011000110000000011000110000000", "-": "00000000000000011111000000000000000",
    "=": "00000000001111100000111110000000000", "/": "00000000010001000100010001000000000",
    "(": "00010001000100001000010000010000010", ")": "01000001000001000010000100010001000",
    ">": "10000010000010000010001000100010000", "%": "11000110010001000100010001001100011",
    "_": "00000000000000000000000000000011111", "+": "00000001000010011111001000010000000",
    ",": "00000000000000000000001100010001000", "x": "00000000001000101010001000101010001",
}


class Canvas:
    def __init__(self, w: int, h: int, bg: Color = (255, 255, 255)):
        self.w, self.h = w, h
        self.px = bytearray(bytes(bg) * (w * h))

    def rect(self, x0: int, y0: int, x1: int, y1: int, c: Color) -> None:
        x0, x1 = max(0, min(x0, x1)), min(self.w, max(x0, x1))
        y0, y1 = max(0, min(y0, y1)), min(self.h, max(y0, y1))
        row = bytes(c) * (x1 - x0)
        for y in range(y0, y1):
            o = (y * self.w + x0) * 3
            self.px[o:o + len(row)] = row

    def frame(self, x0: int, y0: int, x1: int, y1: int, c: Color) -> None:
        self.rect(x0, y0, x1, y0 + 1, c)
        self.rect(x0, y1 - 1, x1, y1, c)
        self.rect(x0, y0, x0 + 1, y1, c)
        self.rect(x1 - 1, y0, x1, y1, c)

    def text(self, x: int, y: int, s: str, c: Color = (0, 0, 0), scale: int = 1) -> int:
        """Draws `s`; returns the x after the last glyph."""
        for ch in s.upper():
            g = _FONT.get(ch, _FONT[" "])
            for r in range(7):
                for col in range(5):
                    if g[r * 5 + col] == "1":
                        self.rect(x + col * scale, y + r * scale, x + (col + 1) * scale,
                                  y + (r + 1) * scale, c)
            x += 6 * scale
        return x

    def save(self, path: str) -> None:
        raw = bytearray()
        stride = self.w * 3
        for y in range(self.h):
            raw.append(0)
            raw += self.px[y * stride:(y + 1) * stride]

        def chunk(tag: bytes, data: bytes) -> bytes:
            return (struct.pack(">I", len(data)) + tag + data +
                    struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF))

        png = b"\x89PNG\r\n\x1a\n"
        png += chunk(b"IHDR", struct.pack(">IIBBBBB", self.w, self.h, 8, 2, 0, 0, 0))
        png += chunk(b"IDAT", zlib.compress(bytes(raw), 6))
        png += chunk(b"IEND", b"")
        with open(path, "wb") as f:
            f.write(png)
