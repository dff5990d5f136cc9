"""Seeded random-init KataGo nets, written in KataGo's `.bin` model format.

The token order and gates follow the reference's model parser, `tools/bin2onnx/bin2onnx.py`
(`parse_model` :1009, `parse_trunk` :718, `parse_policy_head` :774, `parse_value_head` :833, the layer parsers
:138-260 and the transformer parsers :406-560). Float arrays are written as `@BIN@` + little-endian float32
(`ModelReader.floats`, bin2onnx.py:92-125); conv weights in file order (y, x, ic, oc) (bin2onnx.py:160-161) and
matmul weights in (ic, oc) (bin2onnx.py:216-217).

Weights: He-normal convs (std sqrt(2 / (k*k*ic))), batch norm mean 0 / var 1 / gamma ~ U(0.8, 1.2) / beta 0,
linears std 1/sqrt(fan_in). The last layer of every residual branch (final conv, post conv, attention output
projection, FFN second linear) is additionally scaled by 1/sqrt(L), L = residual adds on the trunk (fixup-style),
so that activations stay O(1) through 18 blocks in f16 instead of doubling their variance per block.

`NETS` holds the benchmark configurations (b10c128, b18c384nbt, b10c384h6, tf3-b11c768) and small test nets that
exercise every block kind, activation, trunk-tip norm, RoPE flavour and policy-channel count the parser accepts.
"""

from __future__ import annotations

import gzip
import io
import struct
from dataclasses import dataclass, field
from typing import List, Optional, Union

import numpy as np

ACT_IDENTITY = "ACTIVATION_IDENTITY"
ACT_RELU = "ACTIVATION_RELU"
ACT_MISH = "ACTIVATION_MISH"
ACT_SILU = "ACTIVATION_SILU"


# ---------------------------------------------------------------------------------------------------------------
# Architecture specs
# ---------------------------------------------------------------------------------------------------------------

@dataclass
class Ordinary:
    """ordinary_block: preBN-act-conv(k) c->c, midBN-act-conv(k) c->c (bin2onnx.py:232-249)."""
    k: int = 3


@dataclass
class GPool:
    """gpool_block: regular conv c->regular, gpool conv c->gpool, gpool BN-act, 3*gpool->regular matmul,
    midBN-act, final conv regular->c (bin2onnx.py:270-302)."""
    regular: int
    gpool: int
    k: int = 3


@dataclass
class Nested:
    """nested_bottleneck_block: preBN-act-1x1 c->mid, inner stack at mid, postBN-act-1x1 mid->c
    (bin2onnx.py:321-338)."""
    mid: int
    blocks: list


@dataclass
class Attention:
    """transformer_attention_block (bin2onnx.py:489-524)."""
    heads: int
    kv_heads: int
    head_dim: int = 64
    v_head_dim: int = 64
    rope: str = "fixed"          # "none", "fixed", "learnable"
    rope_theta: float = 100.0


@dataclass
class FFN:
    """transformer_ffn_block with SwiGLU (bin2onnx.py:543-560)."""
    ffn: int


Block = Union[Ordinary, GPool, Nested, Attention, FFN]


@dataclass
class NetSpec:
    name: str
    version: int
    trunk: int
    blocks: List[Block]
    stem_k: int = 5
    act: str = ACT_MISH              # activation of every act layer (v>=11; relu implied for older)
    tip: str = "bn"                  # "bn", "rms", "rms_spatial"
    p1: int = 32
    g1: int = 32
    v1: int = 32
    v2: int = 64
    policy_channels: Optional[int] = None   # v17 only (2 or 4); else implied by the version
    meta_encoder: int = 0            # 0, or 1 (SGF metadata encoder, 192 inputs)
    meta_hidden: int = 32
    regular_hdr: int = 0             # trunk header numbers that only matter to the parser
    gpool_hdr: int = 0
    mid_hdr: int = 0
    eps: float = 1e-5
    rms_eps: float = 1e-6
    input_channels: int = 22
    global_channels: int = 19


def _nested(mid, inner):
    return Nested(mid=mid, blocks=inner)


def b10c128() -> NetSpec:
    """g170e-b10c128-like classic residual net, model version 8 (relu implied, 1 policy channel, 4 score values),
    10 blocks at 128 channels, global pooling in blocks 3/6/9 (1-based), 5x5 stem."""
    blocks: List[Block] = []
    for i in range(10):
        blocks.append(GPool(regular=96, gpool=32) if i in (2, 5, 8) else Ordinary())
    return NetSpec("b10c128", 8, 128, blocks, stem_k=5, act=ACT_RELU, v2=32,
                   regular_hdr=96, gpool_hdr=32, mid_hdr=128)


def b18c384nbt() -> NetSpec:
    """kata1-b18c384nbt-like nested-bottleneck net, model version 14 (mish, 2 policy channels, 6 score values):
    18 blocks of 1x1 384->192, two inner residual pairs of 3x3 convs at 192, 1x1 192->384. Every third block's
    first inner block is a gpool block (regular 192->128, gpool 192->64). 5x5 stem."""
    blocks: List[Block] = []
    for i in range(18):
        first = GPool(regular=128, gpool=64) if i % 3 == 2 else Ordinary()
        blocks.append(_nested(192, [first, Ordinary()]))
    return NetSpec("b18c384nbt", 14, 384, blocks, stem_k=5, act=ACT_MISH, v2=80,
                   regular_hdr=192, gpool_hdr=64, mid_hdr=192)


def b10c384h6() -> NetSpec:
    """Transformer net, model version 17: 10 x (attention with 6 heads of 64 and learnable 2D RoPE, SwiGLU FFN of
    width 1024) at 384 channels, SiLU heads, per-position RMSNorm trunk tip, 3x3 stem."""
    blocks: List[Block] = []
    for _ in range(10):
        blocks.append(Attention(heads=6, kv_heads=6, rope="learnable"))
        blocks.append(FFN(ffn=1024))
    return NetSpec("b10c384h6", 17, 384, blocks, stem_k=3, act=ACT_SILU, tip="rms", policy_channels=2,
                   v2=64, regular_hdr=384, gpool_hdr=64, mid_hdr=384)


def tf3_b11c768() -> NetSpec:
    """tf3-b11c768-like transformer net, model version 17: 11 x (attention with 12 heads of 64 and fixed-theta
    2D RoPE, SwiGLU FFN of width 2048) at 768 channels, spatial RMSNorm trunk tip, 4 policy channels."""
    blocks: List[Block] = []
    for _ in range(11):
        blocks.append(Attention(heads=12, kv_heads=12, rope="fixed", rope_theta=100.0))
        blocks.append(FFN(ffn=2048))
    return NetSpec("tf3-b11c768", 17, 768, blocks, stem_k=3, act=ACT_SILU, tip="rms_spatial", policy_channels=4,
                   p1=48, g1=48, v1=48, v2=96, regular_hdr=768, gpool_hdr=64, mid_hdr=768)


# Small nets for parity tests: every block kind and option, cheap enough for the CPU oracle.
def tiny_resnet() -> NetSpec:
    return NetSpec("tiny-resnet", 8, 32, [Ordinary(), GPool(regular=24, gpool=16), Ordinary()],
                   stem_k=5, act=ACT_RELU, p1=16, g1=16, v1=16, v2=16)


def tiny_nbt() -> NetSpec:
    blocks = [_nested(32, [Ordinary(), Ordinary()]), _nested(32, [GPool(regular=16, gpool=16), Ordinary()])]
    return NetSpec("tiny-nbt", 14, 64, blocks, stem_k=5, act=ACT_MISH, p1=16, g1=16, v1=16, v2=32)


def tiny_v15_meta() -> NetSpec:
    blocks = [_nested(32, [GPool(regular=16, gpool=16), Ordinary()]), Ordinary()]
    return NetSpec("tiny-v15-meta", 15, 64, blocks, stem_k=3, act=ACT_MISH, p1=16, g1=16, v1=16, v2=32,
                   meta_encoder=1, meta_hidden=32)


def tiny_tf_learn() -> NetSpec:
    blocks = [Attention(heads=4, kv_heads=2, head_dim=16, v_head_dim=16, rope="learnable"), FFN(ffn=96),
              Ordinary(), Attention(heads=2, kv_heads=2, head_dim=32, v_head_dim=32, rope="fixed"), FFN(ffn=64)]
    return NetSpec("tiny-tf-learn", 17, 64, blocks, stem_k=3, act=ACT_SILU, tip="rms", policy_channels=4,
                   p1=16, g1=16, v1=16, v2=16)


def tiny_tf_spatial() -> NetSpec:
    blocks = [_nested(64, [Attention(heads=2, kv_heads=1, head_dim=32, v_head_dim=32, rope="none"), FFN(ffn=128)]),
              GPool(regular=32, gpool=16)]
    return NetSpec("tiny-tf-spatial", 17, 64, blocks, stem_k=3, act=ACT_SILU, tip="rms_spatial", policy_channels=2,
                   p1=16, g1=16, v1=16, v2=16)


def small_nbt() -> NetSpec:
    """b18c384nbt's shapes (384 trunk, 192 mid, 128+64 gpool) with 3 blocks: the GPU kernels' real tile shapes at
    a depth the CPU oracle finishes in seconds."""
    blocks: List[Block] = []
    for i in range(3):
        first = GPool(regular=128, gpool=64) if i % 3 == 2 else Ordinary()
        blocks.append(_nested(192, [first, Ordinary()]))
    return NetSpec("small-nbt", 14, 384, blocks, stem_k=5, act=ACT_MISH, v2=80)


def wide_nbt() -> NetSpec:
    """256-channel trunk: the CTA-pair GEMM's 256-wide tiles (windowed 3x3, the gpool conv's two segments
    192 + 64, the 1x1 post conv with a residual) and 128-wide tiles (the nested block's 1x1 pre conv and 3x3)."""
    blocks: List[Block] = [Ordinary(), GPool(regular=192, gpool=64), _nested(128, [Ordinary()])]
    return NetSpec("wide-nbt", 14, 256, blocks, stem_k=3, act=ACT_MISH, v2=48)


def small_tf() -> NetSpec:
    """b10c384h6's shapes with 2 blocks."""
    blocks: List[Block] = []
    for _ in range(2):
        blocks.append(Attention(heads=6, kv_heads=6, rope="learnable"))
        blocks.append(FFN(ffn=1024))
    return NetSpec("small-tf", 17, 384, blocks, stem_k=3, act=ACT_SILU, tip="rms", policy_channels=2, v2=64)


def gqa_tf() -> NetSpec:
    """Grouped-query attention at head dim 64 (the tensor-core attention kernel's KV-head mapping): 6 query heads
    over 2 KV heads, then 4 over 1, fixed-theta RoPE; spatial RMSNorm trunk tip at a width of 384 (the row-parallel
    tip kernels)."""
    blocks: List[Block] = [Attention(heads=6, kv_heads=2, rope="fixed", rope_theta=100.0), FFN(ffn=512),
                           Attention(heads=4, kv_heads=1, rope="learnable"), FFN(ffn=256)]
    return NetSpec("gqa-tf", 17, 384, blocks, stem_k=3, act=ACT_SILU, tip="rms_spatial", policy_channels=2, v2=64)


NETS = {
    "b10c128": b10c128,
    "b18c384nbt": b18c384nbt,
    "b10c384h6": b10c384h6,
    "tf3-b11c768": tf3_b11c768,
    "tiny-resnet": tiny_resnet,
    "tiny-nbt": tiny_nbt,
    "tiny-v15-meta": tiny_v15_meta,
    "tiny-tf-learn": tiny_tf_learn,
    "tiny-tf-spatial": tiny_tf_spatial,
    "small-nbt": small_nbt,
    "small-tf": small_tf,
    "wide-nbt": wide_nbt,
    "gqa-tf": gqa_tf,
}


# ---------------------------------------------------------------------------------------------------------------
# Writer
# ---------------------------------------------------------------------------------------------------------------

class _Writer:
    def __init__(self, spec: NetSpec, seed: int):
        self.spec = spec
        self.rng = np.random.default_rng(seed)
        self.out = io.BytesIO()
        self.n_res = _count_residuals(spec.blocks)

    # tokens -------------------------------------------------------------------------------------------------
    def tok(self, *items):
        for it in items:
            if isinstance(it, float):
                s = repr(float(np.float32(it)))
            else:
                s = str(it)
            self.out.write(s.encode("ascii"))
            self.out.write(b" ")
        self.out.write(b"\n")

    def floats(self, arr: np.ndarray):
        a = np.ascontiguousarray(arr, dtype="<f4").reshape(-1)
        self.out.write(b"@BIN@")
        self.out.write(a.tobytes())
        self.out.write(b"\n")

    # layers -------------------------------------------------------------------------------------------------
    def conv(self, name, k, ic, oc, scale=1.0):
        self.tok(name, k, k, ic, oc, 1, 1)
        std = np.sqrt(2.0 / (k * k * ic)) * scale
        w = self.rng.normal(0.0, std, size=(k, k, ic, oc)).astype(np.float32)  # file order y,x,ic,oc
        self.floats(w)

    def bn(self, name, c):
        self.tok(name, c, self.spec.eps, 1, 1)
        self.floats(np.zeros(c, np.float32))                                   # mean
        self.floats(np.ones(c, np.float32))                                    # variance
        self.floats(self.rng.uniform(0.8, 1.2, size=c).astype(np.float32))     # scale (gamma)
        self.floats(np.zeros(c, np.float32))                                   # bias (beta)

    def act(self, name, kind=None):
        if self.spec.version >= 11:
            self.tok(name, kind or self.spec.act)
        else:
            self.tok(name)

    def matmul(self, name, ic, oc, scale=1.0):
        self.tok(name, ic, oc)
        w = self.rng.normal(0.0, scale / np.sqrt(ic), size=(ic, oc)).astype(np.float32)
        self.floats(w)

    def matbias(self, name, c):
        self.tok(name, c)
        self.floats(self.rng.uniform(-0.1, 0.1, size=c).astype(np.float32))

    def tf_rms(self, name, c):
        self.tok(name, c, self.spec.rms_eps)
        self.floats(self.rng.uniform(0.8, 1.2, size=c).astype(np.float32))

    # blocks -------------------------------------------------------------------------------------------------
    def res_scale(self):
        return 1.0 / np.sqrt(max(1, self.n_res))

    def block(self, b: Block, name: str, c: int):
        if isinstance(b, Ordinary):
            self.tok("ordinary_block")
            self.tok(name)
            self.bn(name + "/norm1", c)
            self.act(name + "/act1")
            self.conv(name + "/w1", b.k, c, c)
            self.bn(name + "/norm2", c)
            self.act(name + "/act2")
            self.conv(name + "/w2", b.k, c, c, scale=self.res_scale())
        elif isinstance(b, GPool):
            self.tok("gpool_block")
            self.tok(name)
            self.bn(name + "/norm1", c)
            self.act(name + "/act1")
            self.conv(name + "/w1a", b.k, c, b.regular)
            self.conv(name + "/w1b", b.k, c, b.gpool)
            self.bn(name + "/norm1b", b.gpool)
            self.act(name + "/act1b")
            self.matmul(name + "/w1r", 3 * b.gpool, b.regular)
            self.bn(name + "/norm2", b.regular)
            self.act(name + "/act2")
            self.conv(name + "/w2", b.k, b.regular, c, scale=self.res_scale())
        elif isinstance(b, Nested):
            self.tok("nested_bottleneck_block")
            self.tok(name, len(b.blocks))
            self.bn(name + "/normpre", c)
            self.act(name + "/actpre")
            self.conv(name + "/convpre", 1, c, b.mid)
            for i, ib in enumerate(b.blocks):
                self.block(ib, f"{name}/blockstack/b{i}", b.mid)
            self.bn(name + "/normpost", b.mid)
            self.act(name + "/actpost")
            self.conv(name + "/convpost", 1, b.mid, c, scale=self.res_scale())
        elif isinstance(b, Attention):
            self.tok("transformer_attention_block")
            use_rope = b.rope != "none"
            learn = b.rope == "learnable"
            self.tok(name, b.heads, b.kv_heads, b.head_dim, b.v_head_dim, int(use_rope), int(learn))
            self.tf_rms(name + "/ln", c)
            self.matmul(name + "/q", c, b.heads * b.head_dim)
            self.matmul(name + "/k", c, b.kv_heads * b.head_dim)
            self.matmul(name + "/v", c, b.kv_heads * b.v_head_dim)
            self.matmul(name + "/out", b.heads * b.v_head_dim, c, scale=self.res_scale())
            if use_rope:
                if learn:
                    pairs = b.head_dim // 2
                    self.tok(name + "/ropefreqs", b.kv_heads, pairs, 2)
                    # (freqX, freqY) per kv head and pair, spread like a theta=100 table with random signs
                    base = 1.0 / np.power(100.0, np.arange(pairs) / pairs)
                    f = base[None, :, None] * self.rng.uniform(-1.5, 1.5, size=(b.kv_heads, pairs, 2))
                    self.floats(f.astype(np.float32))
                else:
                    self.tok(name + "/ropetheta", b.rope_theta)
        elif isinstance(b, FFN):
            self.tok("transformer_ffn_block")
            self.tok(name, c, b.ffn, 1)
            self.tf_rms(name + "/ln", c)
            self.matmul(name + "/w1", c, b.ffn)
            self.matmul(name + "/wgate", c, b.ffn)
            self.matmul(name + "/w2", b.ffn, c, scale=self.res_scale())
        else:
            raise TypeError(type(b))

    # model --------------------------------------------------------------------------------------------------
    def write(self) -> bytes:
        s = self.spec
        v = s.version
        self.tok(s.name, v, s.input_channels, s.global_channels)
        if v >= 13:
            self.tok(20.0, 20.0, 20.0, 20.0, 40.0, 0.25, 30.0)
        if v >= 15:
            self.tok(s.meta_encoder, 0, 0, 0, 0, 0, 0, 0)
        # trunk header: name numBlocks trunkC midC regularC dilatedC gpoolC [v15+: normKind B..F]
        self.tok("trunk", len(s.blocks), s.trunk, s.mid_hdr or s.trunk, s.regular_hdr or s.trunk, 0,
                 s.gpool_hdr or 32)
        if v >= 15:
            self.tok(0 if s.tip == "bn" else 1, 0, 0, 0, 0, 0)
        self.conv("conv1", s.stem_k, s.input_channels, s.trunk)
        self.matmul("ginputw", s.global_channels, s.trunk)
        if s.meta_encoder:
            self.tok("sgfmeta", 192)
            self.matmul("sgfmeta/mul1", 192, s.meta_hidden)
            self.matbias("sgfmeta/bias1", s.meta_hidden)
            self.act("sgfmeta/act1")
            self.matmul("sgfmeta/mul2", s.meta_hidden, s.meta_hidden)
            self.matbias("sgfmeta/bias2", s.meta_hidden)
            self.act("sgfmeta/act2")
            self.matmul("sgfmeta/mul3", s.meta_hidden, s.trunk, scale=0.5)
        for i, b in enumerate(s.blocks):
            self.block(b, f"rconv{i + 1}", s.trunk)
        if s.tip == "bn":
            self.bn("trunk/norm", s.trunk)
        else:
            # RMSNormLayerDesc: name c eps spatial cgroupSize gamma beta
            self.tok("trunk/rmsnorm", s.trunk, s.rms_eps, 1 if s.tip == "rms_spatial" else 0, 0)
            self.floats(self.rng.uniform(0.8, 1.2, size=s.trunk).astype(np.float32))
            self.floats(self.rng.uniform(-0.1, 0.1, size=s.trunk).astype(np.float32))
        self.act("trunk/act")
        self._policy_head()
        self._value_head()
        return self.out.getvalue()

    def _num_policy(self):
        v = self.spec.version
        if v >= 17:
            return self.spec.policy_channels or 2
        if v == 16:
            return 4
        if v >= 12:
            return 2
        return 1

    def _policy_head(self):
        s = self.spec
        v = s.version
        p = self._num_policy()
        self.tok("policyhead")
        if v >= 17:
            self.tok(p, 0, 0, 0)
        self.conv("p1/w", 1, s.trunk, s.p1)
        self.conv("g1/w", 1, s.trunk, s.g1)
        self.bn("g1/norm", s.g1)
        self.act("g1/act")
        self.matmul("matmulg2w", 3 * s.g1, s.p1)
        self.bn("p1/norm", s.p1)
        self.act("p1/act")
        self.conv("p2/w", 1, s.p1, p)
        if v >= 15:
            self.matmul("matmulpass", 3 * s.g1, s.p1)
            self.matbias("matbiaspass", s.p1)
            self.act("passact")
            self.matmul("matmulpass2", s.p1, p)
        else:
            self.matmul("matmulpass", 3 * s.g1, p)

    def _value_head(self):
        s = self.spec
        v = s.version
        self.tok("valuehead")
        if v >= 17:
            self.tok(0, 0, 0)
        self.conv("v1/w", 1, s.trunk, s.v1)
        self.bn("v1/norm", s.v1)
        self.act("v1/act")
        self.matmul("v2/w", 3 * s.v1, s.v2)
        self.matbias("v2/b", s.v2)
        self.act("v2/act")
        self.matmul("v3/w", s.v2, 3)
        self.matbias("v3/b", 3)
        nsv = 6 if v >= 9 else 4 if v >= 8 else 2 if v >= 4 else 1
        self.matmul("sv3/w", s.v2, nsv)
        self.matbias("sv3/b", nsv)
        self.conv("vownership/w", 1, s.v1, 1)


def _count_residuals(blocks) -> int:
    n = 0
    for b in blocks:
        n += 1
        if isinstance(b, Nested):
            n += _count_residuals(b.blocks)
    return n


def write_bin(spec: NetSpec, seed: int) -> bytes:
    """The net `spec` with seeded random weights, as the bytes of a KataGo `.bin` file."""
    return _Writer(spec, seed).write()


def write_bin_gz(spec: NetSpec, seed: int) -> bytes:
    return gzip.compress(write_bin(spec, seed), mtime=0)


def net_bytes(name: str, seed: Optional[int] = None, gz: bool = False) -> bytes:
    """The seeded `.bin` (or `.bin.gz`) bytes of a named net; the default seed is fixed per net name."""
    spec = NETS[name]()
    if seed is None:
        seed = 0xB200 + sum(map(ord, name))
    return write_bin_gz(spec, seed) if gz else write_bin(spec, seed)


# ---------------------------------------------------------------------------------------------------------------
# Algorithmic FLOPs (direct-conv MACs x 2 over the 361 board points; attention QK and PV over 361 x 361)
# ---------------------------------------------------------------------------------------------------------------

def flops_per_eval(spec: NetSpec, area: int = 361) -> dict:
    out = {"conv3x3": 0.0, "conv1x1": 0.0, "stem": 0.0, "linear": 0.0, "attention": 0.0, "heads": 0.0}

    def walk(blocks, c):
        for b in blocks:
            if isinstance(b, Ordinary):
                key = "conv3x3" if b.k == 3 else "stem"
                out[key] += 2 * 2.0 * area * b.k * b.k * c * c
            elif isinstance(b, GPool):
                out["conv3x3"] += 2.0 * area * 9 * c * (b.regular + b.gpool) + 2.0 * area * 9 * b.regular * c
            elif isinstance(b, Nested):
                out["conv1x1"] += 2 * 2.0 * area * c * b.mid
                walk(b.blocks, b.mid)
            elif isinstance(b, Attention):
                out["linear"] += 2.0 * area * c * (b.heads * b.head_dim + 2 * b.kv_heads * b.head_dim)
                out["linear"] += 2.0 * area * b.heads * b.v_head_dim * c
                out["attention"] += 2.0 * area * area * b.heads * (b.head_dim + b.v_head_dim)
            elif isinstance(b, FFN):
                out["linear"] += 2.0 * area * c * b.ffn * 3
    walk(spec.blocks, spec.trunk)
    out["stem"] += 2.0 * area * spec.stem_k ** 2 * spec.input_channels * spec.trunk
    out["heads"] += 2.0 * area * spec.trunk * (spec.p1 + spec.g1 + spec.v1)
    out["total"] = sum(out.values())
    return out
