"""TEST INFRASTRUCTURE — ctypes binding of the CPU oracle (oracle/liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module. It is the checker, never the thing measured or shipped: the
product library (libqwen_b200.so) neither links nor calls it.

The oracle restates the reference's scalar math (native/operator_reference.h,
native/projection_reference.h, native/attention_reference.h, wiring of
native/qwen_model.inc); see oracle/qwen_oracle.cpp for the per-function
citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_oracle.so"


class RsQwenConfig(C.Structure):
    """Mirror of rs_qwen_config (native/mlx_bridge.h:50-53), 132 bytes."""

    _fields_ = [(n, C.c_int32) for n in (
        "hidden layers vocab q_heads kv_heads head_dim key_heads value_heads key_dim "
        "value_dim conv interval experts top intermediate shared group bits context chunk "
        "rope_dims activation_precision layer_group fused_recurrent execution_timing "
        "compiled_decode operator_profile fused_attention validation_mode "
        "validation_interval expert_kernel").split()] + [("epsilon", C.c_float), ("theta", C.c_float)]


assert C.sizeof(RsQwenConfig) == 132


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile (g++ only)."""
    if force or not LIB.exists() or LIB.stat().st_mtime < max(
            (HERE / f).stat().st_mtime for f in ("qwen_oracle.cpp", "fp32_step.cpp", "synth.h", "Makefile")):
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB


def reference_root() -> Path | None:
    """Location of the reference checkout: the QWEN_REFERENCE environment
    variable, else BASELINE.json's "reference_path". None when neither names
    an existing directory (the GPU box has no reference tree)."""
    where = os.environ.get("QWEN_REFERENCE")
    if not where:
        meta = HERE.parent / "BASELINE.json"
        if meta.exists():
            import json

            where = json.loads(meta.read_text()).get("reference_path")
    if where and Path(where).is_dir():
        return Path(where)
    return None


def build_ref() -> Path | None:
    """Compile oracle/_ref/libref_oracle.so from the reference's own oracle
    headers when the reference checkout is present (see reference_root)."""
    root = reference_root()
    ref = root / "native" if root else None
    if ref is None or not (ref / "operator_reference.h").exists():
        return REF_LIB if REF_LIB.exists() else None
    subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)
    return REF_LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(build()))
        L = _lib
        P, D, F, I32, U32, SZ = (C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_float),
                                 C.POINTER(C.c_int32), C.POINTER(C.c_uint32), C.c_size_t)
        L.orc_last_error.restype = C.c_char_p
        L.orc_set_routing_slack.argtypes = [C.c_double]
        L.orc_set_emulation.argtypes = [C.c_int]
        L.orc_state_count.restype = SZ
        L.orc_state_count.argtypes = [C.POINTER(RsQwenConfig)]
        L.orc_model_create.restype = P
        L.orc_model_create.argtypes = [C.POINTER(RsQwenConfig), C.c_uint64, C.c_int]
        L.orc_model_destroy.argtypes = [P]
        L.orc_model_qrows.argtypes = [P, C.c_char_p, SZ, SZ, U32, F, F]
        L.orc_model_vector.argtypes = [P, C.c_char_p, F, SZ]
        L.orc_forward.argtypes = [P, U32, SZ, SZ, F, F, D, D, I32, SZ, I32]
        L.orc_mtp_forward.argtypes = [P, U32, SZ, SZ, D, D, D, D, I32, SZ]
        L.orc_projection.argtypes = [F, U32, F, F, SZ, SZ, SZ, C.c_int, C.c_int, D]
        L.orc_rms.argtypes = [F, F, SZ, SZ, C.c_double, D]
        L.orc_silu.argtypes = [F, SZ, D]
        L.orc_rope.argtypes = [F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double, D]
        L.orc_delta.argtypes = [F] * 8 + [C.c_int] * 6 + [D] * 4
        L.orc_attention.argtypes = [F, F, F] + [C.c_int] * 5 + [D]
        L.orc_routing.argtypes = [F, I32, C.c_int, C.c_int, C.c_int, D, D]
        L.orc_topk.argtypes = [F, SZ, SZ, SZ, I32]
        L.orc_argmax.restype = C.c_int64
        L.orc_argmax.argtypes = [F, SZ]
        L.orc_expert_sort.argtypes = [I32, SZ, SZ, I32, I32, I32, I32]
        L.orc_pack_ragged.argtypes = [SZ] + [I32] * 8 + [C.c_int32, I32, SZ, I32, I32, I32,
                                                          C.POINTER(C.c_int64)]
        L.orc_accept.argtypes = [C.c_uint32, U32, U32, SZ, U32, SZ, SZ, U32, U32, U32, U32]
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t)) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def check(rc: int):
    if rc != 0:
        raise RuntimeError(lib().orc_last_error().decode())


def config(**kw) -> RsQwenConfig:
    c = RsQwenConfig()
    defaults = dict(activation_precision=1, layer_group=1, validation_mode=0,
                    validation_interval=1, chunk=8, group=64, bits=4, epsilon=1e-6,
                    theta=1e7, interval=4, conv=4)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(c, k, v)
    return c


# tiny hybrid decoder (vocab 4096, hidden 256, 4 layers
# [GDN,GDN,GDN,attn], 4q/1kv/64, GDN 4v/2qk/64, conv 4, 16 experts top-2 +
# 1 shared, expert width 128).
def config0(context: int = 512) -> RsQwenConfig:
    return config(hidden=256, layers=4, vocab=4096, q_heads=4, kv_heads=1, head_dim=64,
                  key_heads=2, value_heads=4, key_dim=64, value_dim=64, experts=16, top=2,
                  intermediate=128, shared=128, context=context, rope_dims=16)


# Qwen3-Next-80B-A3B shapes. `layers` may be cut to a
# multiple of 4 for oracle-sized parity cases.
def config1(layers: int = 48, context: int = 32768 + 64, vocab: int = 151936) -> RsQwenConfig:
    return config(hidden=2048, layers=layers, vocab=vocab, q_heads=16, kv_heads=2, head_dim=256,
                  key_heads=16, value_heads=32, key_dim=128, value_dim=128, experts=512, top=10,
                  intermediate=512, shared=512, context=context, rope_dims=64)


class Model:
    """Lazily generated synthetic model (same bytes as rs_qwen_weights_synthetic)."""

    def __init__(self, cfg: RsQwenConfig, seed: int, mtp: bool = False):
        self.cfg = cfg
        self.h = lib().orc_model_create(C.byref(cfg), seed, int(mtp))
        if not self.h:
            raise RuntimeError(lib().orc_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_destroy(self.h)
            self.h = None

    def state_count(self) -> int:
        return lib().orc_state_count(C.byref(self.cfg))

    def qrows(self, name: str, row0: int, n: int, cols: int):
        packed = np.zeros((n, cols // 8), np.uint32)
        sc = np.zeros((n, cols // 64), np.float32)
        bi = np.zeros((n, cols // 64), np.float32)
        check(lib().orc_model_qrows(self.h, name.encode(), row0, n, _p(packed, C.c_uint32),
                                    _p(sc, C.c_float), _p(bi, C.c_float)))
        return packed, sc, bi

    def override(self, name: str, bits: int, group: int, packed, scales, biases):
        """Use rows in another quantization for matrix `name` (orc_model_override)."""
        pk = np.ascontiguousarray(packed, np.uint32)
        sc = np.ascontiguousarray(scales, np.float32)
        bi = np.ascontiguousarray(biases, np.float32)
        L = lib()
        L.orc_model_override.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_uint32),
                                         C.POINTER(C.c_float), C.POINTER(C.c_float)]
        check(L.orc_model_override(self.h, name.encode(), bits, group, _p(pk, C.c_uint32), _p(sc, C.c_float),
                                   _p(bi, C.c_float)))

    def vector(self, name: str, n: int):
        out = np.zeros(n, np.float32)
        check(lib().orc_model_vector(self.h, name.encode(), _p(out, C.c_float), n))
        return out

    def forward(self, tokens, offset: int, old_state=None, hidden: bool = False,
                forced_routing=None):
        """Returns (logits [count, vocab] f64, new_state f32, hidden or None, routing)."""
        c = self.cfg
        tok = np.ascontiguousarray(tokens, np.uint32)
        n = self.state_count()
        new = np.zeros(n, np.float32)
        old = _f32(old_state) if old_state is not None else np.zeros(1, np.float32)
        logits = np.zeros((len(tok), c.vocab), np.float64)
        hid = np.zeros((len(tok), c.hidden), np.float64) if hidden else None
        moe_layers = c.layers
        routed = np.zeros((moe_layers, len(tok), c.top), np.int32)
        forced = None if forced_routing is None else np.ascontiguousarray(forced_routing, np.int32)
        check(lib().orc_forward(self.h, _p(tok, C.c_uint32), len(tok), offset, _p(old, C.c_float),
                                _p(new, C.c_float), _p(logits, C.c_double),
                                _p(hid, C.c_double), _p(forced, C.c_int32),
                                0 if forced is None else forced.size, _p(routed, C.c_int32)))
        return logits, new, hid, routed

    def mtp_forward(self, tokens, offset: int, target_hidden, kv_state, forced_routing=None):
        c = self.cfg
        tok = np.ascontiguousarray(tokens, np.uint32)
        th = np.ascontiguousarray(target_hidden, np.float64)
        logits = np.zeros((len(tok), c.vocab), np.float64)
        hid = np.zeros((len(tok), c.hidden), np.float64)
        forced = None if forced_routing is None else np.ascontiguousarray(forced_routing, np.int32)
        check(lib().orc_mtp_forward(self.h, _p(tok, C.c_uint32), len(tok), offset,
                                    _p(th, C.c_double), _p(kv_state, C.c_double),
                                    _p(logits, C.c_double), _p(hid, C.c_double),
                                    _p(forced, C.c_int32), 0 if forced is None else forced.size))
        return logits, hid


class F32Step:
    """The timed CPU baseline (fp32_step.cpp): an fp32, std::thread-parallel
    batched decode step over the same synthetic weights."""

    def __init__(self, cfg: RsQwenConfig, seed: int, threads: int = 0):
        L = lib()
        if not getattr(L, "_f32_bound", False):
            L.f32_last_error.restype = C.c_char_p
            L.f32_create.restype = C.c_void_p
            L.f32_create.argtypes = [C.POINTER(RsQwenConfig), C.c_uint64, C.c_int]
            L.f32_destroy.argtypes = [C.c_void_p]
            L.f32_threads.argtypes = [C.c_void_p]
            L.f32_set_batch.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_float),
                                        C.c_uint64, C.c_size_t]
            L.f32_step.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_float),
                                   C.POINTER(C.c_double), C.POINTER(C.c_double)]
            L.f32_stage_seconds.argtypes = [C.c_void_p, C.POINTER(C.c_double)]
            L._f32_bound = True
        self.cfg = cfg
        self.h = L.f32_create(C.byref(cfg), seed, threads)
        if not self.h:
            raise RuntimeError(L.f32_last_error().decode())
        self.threads = L.f32_threads(self.h)
        self.n = 0

    def __del__(self):
        if getattr(self, "h", None):
            lib().f32_destroy(self.h)
            self.h = None

    def _check(self, rc):
        if rc:
            raise RuntimeError(lib().f32_last_error().decode())

    def set_batch(self, positions, states=None, seed: int = 0, extra: int = 64):
        pos = np.ascontiguousarray(positions, np.uint32)
        st = None if states is None else np.ascontiguousarray(states, np.float32)
        self.n = len(pos)
        self._check(lib().f32_set_batch(self.h, len(pos), _p(pos, C.c_uint32), _p(st, C.c_float), seed, extra))

    def step(self, tokens, want_logits: bool = False):
        """One decode token per sequence: (sampled, logits or None, seconds in layers, seconds in the head)."""
        tok = np.ascontiguousarray(tokens, np.uint32)
        sampled = np.zeros(self.n, np.uint32)
        logits = np.zeros((self.n, self.cfg.vocab), np.float32) if want_logits else None
        tl, th = C.c_double(), C.c_double()
        self._check(lib().f32_step(self.h, _p(tok, C.c_uint32), _p(sampled, C.c_uint32), _p(logits, C.c_float),
                                   C.byref(tl), C.byref(th)))
        return sampled, logits, tl.value, th.value

    def stage_seconds(self):
        """(DeltaNet mixers, attention mixers, MoE blocks) seconds of the last step."""
        out = (C.c_double * 3)()
        lib().f32_stage_seconds(self.h, out)
        return tuple(out)


def set_routing_slack(slack: float):
    lib().orc_set_routing_slack(slack)


# Error-analysis knobs of the oracle (0 = exact FP64): round a class of values
# the way a 16-bit device datapath stores them (qwen_oracle.cpp, g_emulate).
EMU_WEIGHTS, EMU_ACTIVATIONS, EMU_KV, EMU_ATTN_QP, EMU_HALF = 1, 2, 4, 8, 256


def set_emulation(bits: int):
    lib().orc_set_emulation(int(bits))


def argmax(logits) -> int:
    a = _f32(logits)
    return int(lib().orc_argmax(_p(a, C.c_float), a.size))


def select(logits, allowed):
    """Constrained greedy selection (choices.rs:65-98); raises on the reference's errors."""
    a = _f32(logits)
    ids = np.ascontiguousarray(allowed, np.uint32)
    L = lib()
    L.orc_select.restype = C.c_int64
    L.orc_select.argtypes = [C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_uint32), C.c_size_t]
    r = L.orc_select(_p(a, C.c_float), a.size, _p(ids, C.c_uint32), ids.size)
    if r < 0:
        raise RuntimeError(L.orc_last_error().decode())
    return int(r)


def topk(logits, top: int):
    a = _f32(logits)
    rows, experts = a.shape
    idx = np.zeros((rows, top), np.int32)
    check(lib().orc_topk(_p(a, C.c_float), rows, experts, top, _p(idx, C.c_int32)))
    return idx


def expert_sort(ids, n_experts: int):
    a = np.ascontiguousarray(ids, np.int32).ravel()
    counts = np.zeros(n_experts, np.int32)
    offsets = np.zeros(n_experts + 1, np.int32)
    perm = np.zeros(a.size, np.int32)
    inv = np.zeros(a.size, np.int32)
    check(lib().orc_expert_sort(_p(a, C.c_int32), a.size, n_experts, _p(counts, C.c_int32),
                                _p(offsets, C.c_int32), _p(perm, C.c_int32), _p(inv, C.c_int32)))
    return counts, offsets, perm, inv


def accept(initial: int, draft, rows, eos, remaining: int):
    d = np.ascontiguousarray(draft, np.uint32)
    r = np.ascontiguousarray(rows, np.uint32)
    e = np.ascontiguousarray(eos, np.uint32)
    emitted = np.zeros(len(d) + 1, np.uint32)
    ne, acc, term = (np.zeros(1, np.uint32) for _ in range(3))
    check(lib().orc_accept(initial, _p(d, C.c_uint32), _p(r, C.c_uint32), len(d),
                           _p(e, C.c_uint32), len(e), remaining, _p(emitted, C.c_uint32),
                           _p(ne, C.c_uint32), _p(acc, C.c_uint32), _p(term, C.c_uint32)))
    return list(emitted[: ne[0]]), int(acc[0]), bool(term[0])


def pack_ragged(position, count, parent_row, child_row, n_shared, new_off, n_new, new_pages,
                page_size, block_table):
    n = len(position)
    i32 = lambda a: np.ascontiguousarray(a, np.int32)  # noqa: E731
    position, count, parent_row, child_row, n_shared, new_off, n_new, new_pages = map(
        i32, (position, count, parent_row, child_row, n_shared, new_off, n_new, new_pages))
    bt = np.ascontiguousarray(block_table, np.int32).copy()
    T = int(count.sum())
    cu = np.zeros(n + 1, np.int32)
    tseq = np.zeros(T, np.int32)
    tpos = np.zeros(T, np.int32)
    slots = np.zeros(T, np.int64)
    check(lib().orc_pack_ragged(n, *(_p(a, C.c_int32) for a in (
        position, count, parent_row, child_row, n_shared, new_off, n_new, new_pages)),
        page_size, _p(bt, C.c_int32), bt.shape[1], _p(cu, C.c_int32), _p(tseq, C.c_int32),
        _p(tpos, C.c_int32), slots.ctypes.data_as(C.POINTER(C.c_int64))))
    return cu, tseq, tpos, slots, bt


def f64(n):
    return np.zeros(n, np.float64)


def call(name: str, *args):
    check(getattr(lib(), name)(*args))


def ptr(a, t=C.c_float):
    return _p(a, t)
