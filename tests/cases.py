"""Parity case tables.

FULL_CASES is the reference's full-kernel problem matrix
(tests/test_configs.hpp:19-102 of poyenc/fmha_native): the same 63 rows,
names and fields {name, b, h, s, d, kv_heads, kv_seq, mask, lse, varlen},
kept identical so a reference user recognises every case.  Inputs come from
the reference generator (glibc srand(42), buffers.cpp:99-127) in the
reference oracle layouts: BHSD dense, [H,total,D] varlen.

BASELINE_CASES are the five north-star configurations.
"""
from __future__ import annotations

import collections

Case = collections.namedtuple("Case", "name b h s d kv_heads kv_seq mask lse varlen")


def _c(name, b, h, s, d, kv_heads=0, kv_seq=0, mask=0, lse=0, opt=0, varlen=()):
    return Case(name, b, h, s, d, kv_heads, kv_seq, mask, lse, tuple(varlen))


FULL_CASES = [
    # D64 smoke
    _c("D64Smoke1", 2, 2, 512, 64, 0, 0, 0, 0, 0),
    _c("D64Smoke2", 1, 1, 256, 64, 0, 0, 0, 0, 0),
    _c("D64Smoke3", 2, 4, 1024, 64, 0, 0, 0, 0, 0),
    _c("D64Smoke4", 1, 8, 2048, 64, 0, 0, 0, 0, 0),
    # feature combos
    _c("D64MaskLse", 2, 4, 1024, 64, 0, 0, 1, 1, 0),
    _c("D64GqaMask", 2, 8, 1024, 64, 2, 0, 1, 0, 0),
    _c("D64MqaMaskLse", 2, 8, 1024, 64, 1, 0, 1, 1, 0),
    _c("D64AsymSqLtSkvMaskLse", 1, 8, 512, 64, 0, 1024, 1, 1, 0),
    _c("D64AsymSqGtSkvMask", 1, 4, 1024, 64, 0, 512, 1, 0, 0),
    _c("D64KitchenSink", 2, 8, 1024, 64, 2, 2048, 1, 1, 0),
    # edge cases
    _c("D64EdgeS300MaskLse", 1, 2, 300, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS300GqaMask", 1, 4, 300, 64, 2, 0, 1, 0, 0),
    _c("D64EdgeS255", 1, 2, 255, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS255MaskLse", 1, 2, 255, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS33MaskLse", 1, 2, 33, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS33MqaMask", 1, 2, 33, 64, 1, 0, 1, 0, 0),
    _c("D64EdgeS17MaskLse", 1, 1, 17, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS17GqaMask", 1, 4, 17, 64, 2, 0, 1, 0, 0),
    _c("D64EdgeS16", 1, 1, 16, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeScale", 1, 1, 8192, 64, 0, 0, 1, 1, 0),
    # varlen
    _c("D64VarlenMask", 4, 4, 1024, 64, 0, 0, 1, 0, 0, (512, 256, 1024, 128)),
    _c("D64VarlenGqaMask", 2, 8, 512, 64, 2, 0, 1, 0, 0, (512, 256)),
    _c("D64VarlenEdgeMaskLse", 2, 2, 300, 64, 0, 0, 1, 1, 0, (300, 33)),
    _c("D64VarlenMqaMaskLse", 4, 8, 1024, 64, 1, 0, 1, 1, 0, (1024, 512, 256, 128)),
    # feature variants
    _c("D64MaskOnly", 2, 4, 1024, 64, 0, 0, 1, 0, 0),
    _c("D64LseOnly", 2, 4, 1024, 64, 0, 0, 0, 1, 0),
    _c("D64GqaAsymMaskLse", 1, 8, 512, 64, 2, 1024, 1, 1, 0),
    _c("D64MqaAsymMask", 1, 8, 1024, 64, 1, 512, 1, 0, 0),
    # boundary / misc
    _c("D64EdgeS300", 1, 2, 300, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS256", 1, 2, 256, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS33", 1, 2, 33, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS17", 1, 1, 17, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeKvseq0", 1, 1, 256, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS1", 1, 1, 1, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS2Mask", 1, 2, 2, 64, 0, 0, 1, 0, 0),
    _c("D64EdgeS31", 1, 2, 31, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS32", 1, 2, 32, 64, 0, 0, 1, 0, 0),
    _c("D64EdgeS64MaskLse", 1, 4, 64, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS257Mask", 1, 2, 257, 64, 0, 0, 1, 0, 0),
    _c("D64H3Mask", 2, 3, 512, 64, 0, 0, 1, 0, 0),
    _c("D64H6GqaMask", 1, 6, 1024, 64, 3, 0, 1, 0, 0),
    _c("D64GqaRatio8MaskLse", 1, 16, 512, 64, 2, 0, 1, 1, 0),
    _c("D64GqaNomask", 2, 8, 1024, 64, 2, 0, 0, 0, 0),
    _c("D64VarlenNomask", 2, 4, 512, 64, 0, 0, 0, 0, 0, (512, 256)),
    _c("D64EdgeKvseq1", 1, 2, 256, 64, 0, 1, 0, 0, 0),
    _c("D64AsymLongContext", 1, 4, 64, 64, 0, 4096, 1, 1, 0),
    _c("D64VarlenTinyMaskLse", 4, 2, 512, 64, 0, 0, 1, 1, 0, (1, 512, 32, 256)),
    _c("D64B8Mask", 8, 4, 512, 64, 0, 0, 1, 0, 0),
    # tile boundary
    _c("D64EdgeS128", 1, 2, 128, 64, 0, 0, 0, 0, 0),
    _c("D64EdgeS128MaskLse", 1, 4, 128, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeS65MaskLse", 1, 2, 65, 64, 0, 0, 1, 1, 0),
    _c("D64EdgeAsymS128Sk65Mask", 1, 2, 128, 64, 0, 65, 1, 0, 0),
    # feature combos (gaps)
    _c("D64GqaLseNomask", 2, 8, 512, 64, 2, 0, 0, 1, 0),
    _c("D64VarlenGqaMaskLse", 2, 8, 512, 64, 2, 0, 1, 1, 0, (512, 256)),
    _c("D64VarlenLseNomask", 2, 4, 512, 64, 0, 0, 0, 1, 0, (512, 256)),
    _c("D64VarlenAsymMask", 2, 4, 256, 64, 0, 512, 1, 0, 0, (256, 128)),
    # causal full-tile-skip coverage
    _c("D64CausalDeepSquare", 1, 2, 768, 64, 0, 0, 1, 0, 0),
    _c("D64CausalDeepSquareLse", 1, 2, 768, 64, 0, 0, 1, 1, 0),
    _c("D64CausalRaggedTail", 1, 2, 832, 64, 0, 0, 1, 0, 0),
    _c("D64CausalDeepRagged", 1, 2, 1100, 64, 0, 0, 1, 0, 0),
    _c("D64CausalShift128", 1, 2, 256, 64, 0, 384, 1, 0, 0),
    _c("D64CausalShift64", 1, 2, 256, 64, 0, 320, 1, 0, 0),
    _c("D64CausalGqaDeepRagged", 1, 8, 900, 64, 2, 0, 1, 0, 0),
]
assert len(FULL_CASES) == 63
