"""SentencePiece precompiled character map (the normaliser of Unigram / SPM tokenizers).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tokenizer/PrecompiledCharsMap.java:1-142.
Blob layout (SentencePiece normalizer): uint32 little-endian trie size in bytes, a Darts double-array trie of
uint32 units over UTF-8 bytes, then NUL-terminated replacement strings.  Normalisation walks the input left to
right, takes the longest prefix that the trie maps, emits its replacement, and otherwise copies one character.
Unit fields: has_leaf = bit 8, value = low 31 bits, label = bits 0-7 plus bit 31,
offset = (unit >> 10) << ((unit & (1 << 9)) >> 6).
"""
from __future__ import annotations

import struct
from typing import List, Optional, Tuple


class PrecompiledCharsMap:
    def __init__(self, blob: bytes):
        self.units: List[int] = []
        self.normalized = b""
        if len(blob) < 4:
            return
        (trie_size,) = struct.unpack("<I", blob[:4])
        trie = blob[4:4 + trie_size]
        self.units = list(struct.unpack(f"<{len(trie) // 4}I", trie[:len(trie) // 4 * 4]))
        self.normalized = blob[4 + trie_size:]

    @staticmethod
    def _offset(u: int) -> int:
        return (u >> 10) << ((u & (1 << 9)) >> 6)

    @staticmethod
    def _label(u: int) -> int:
        return u & ((1 << 31) | 0xFF)

    @staticmethod
    def _has_leaf(u: int) -> bool:
        return ((u >> 8) & 1) == 1

    @staticmethod
    def _value(u: int) -> int:
        return u & ((1 << 31) - 1)

    def longest_match(self, data: bytes, start: int) -> Optional[Tuple[int, int]]:
        """-> (match length in bytes, offset into the replacement blob) of the longest prefix."""
        if not self.units:
            return None
        units = self.units
        pos = 0
        pos ^= self._offset(units[pos])
        best = None
        for i in range(start, len(data)):
            c = data[i]
            pos ^= c
            if pos >= len(units):
                break
            u = units[pos]
            if self._label(u) != c:
                break
            pos ^= self._offset(u)
            if self._has_leaf(u):
                if pos >= len(units):
                    break
                best = (i - start + 1, self._value(units[pos]))
        return best

    def normalize(self, text: str) -> str:
        if not self.units:
            return text
        data = text.encode("utf-8")
        out = bytearray()
        i = 0
        while i < len(data):
            m = self.longest_match(data, i)
            if m is not None:
                length, off = m
                end = self.normalized.find(b"\0", off)
                out += self.normalized[off:end if end >= 0 else len(self.normalized)]
                i += length
            else:
                b = data[i]
                n = 1 if b < 0x80 else 2 if b >> 5 == 0x6 else 3 if b >> 4 == 0xE else 4
                out += data[i:i + n]
                i += n
        return out.decode("utf-8", errors="replace")
