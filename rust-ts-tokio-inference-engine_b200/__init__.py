"""Host-side binding of the B200 ragged hybrid-Qwen decode step.

The product is the C-ABI library ``_lib/libqwen_b200.so`` (CUDA, sm_100a). This
module binds it with ctypes the same way the reference's Rust executor binds
its native bridge (src/serving/native_device.rs:1087-1207): same symbols, same
argument meaning, and the same error convention (0 = ok, -1 = error with a
message, surfaced here as ``NativeError``). There is no CPU path: loading
fails loudly when the library is missing, and creating a session fails on a
machine without a B200.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "_lib" / "libqwen_b200.so"

RAGGED_SAMPLED = 1
RAGGED_LOGITS = 2
RAGGED_ALL_ROWS = 4
RAGGED_HIDDEN = 8
RAGGED_CONSUME = 16
STATS_COUNT = 17 + 19 * 3


class NativeError(RuntimeError):
    """A native call returned -1 (native/mlx_bridge.cpp:19-31 convention)."""


class RsQwenConfig(C.Structure):
    """rs_qwen_config (native/mlx_bridge.h:50-53)."""

    _fields_ = [(n, C.c_int32) for n in (
        "hidden layers vocab q_heads kv_heads head_dim key_heads value_heads key_dim "
        "value_dim conv interval experts top intermediate shared group bits context chunk "
        "rope_dims activation_precision layer_group fused_recurrent execution_timing "
        "compiled_decode operator_profile fused_attention validation_mode "
        "validation_interval expert_kernel").split()] + [("epsilon", C.c_float), ("theta", C.c_float)]


class RsQwenLayer(C.Structure):
    _fields_ = [("index", C.c_uint32), ("mixer", C.c_uint32)]


class StateId(C.Structure):
    """StateId {owner, slot, generation, position, bytes} (native/state_table.h:11-13)."""

    _fields_ = [(n, C.c_uint64) for n in ("owner", "slot", "generation", "position", "bytes")]

    def astuple(self):
        return (self.owner, self.slot, self.generation, self.position, self.bytes)


assert C.sizeof(RsQwenConfig) == 132 and C.sizeof(StateId) == 40

_P, _SZ, _U32P, _F32P, _I32P = C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_float), C.POINTER(C.c_int32)
_SIDP, _ERR = C.POINTER(StateId), C.c_char_p

# symbol -> (restype, argtypes); the declarations of include/qwen_b200.h
SIGNATURES = {
    "rs_mlx_version": (C.c_char_p, []),
    "rs_qwen_state_count": (_SZ, [C.POINTER(RsQwenConfig)]),
    "rs_mlx_weights_create": (_P, [_ERR, _SZ]),
    "rs_mlx_weights_destroy": (None, [_P]),
    "rs_mlx_weights_load": (C.c_int, [_P, C.c_char_p, _ERR, _SZ]),
    "rs_qwen_quant": (C.c_int, [_P, C.c_char_p, C.c_int, C.c_int, _ERR, _SZ]),
    "rs_mlx_weight_bytes": (C.c_int, [_P, C.c_char_p, _I32P, _SZ, C.c_int, _SZ, C.POINTER(C.c_uint8), _SZ, _ERR, _SZ]),
    "rs_qwen_weights_synthetic": (C.c_int, [_P, C.POINTER(RsQwenConfig), C.c_uint64, C.c_int, _ERR, _SZ]),
    "rs_qwen_forward": (C.c_int, [_P, C.c_int, C.POINTER(RsQwenConfig), C.POINTER(RsQwenLayer), _SZ, _U32P, _SZ, _SZ,
                                  _F32P, _SZ, _F32P, _SZ, _F32P, _SZ, C.c_int, _U32P, _SZ, _F32P, _SZ, _ERR, _SZ]),
    "rs_mlx_create": (_P, [C.c_int, _ERR, _SZ]),
    "rs_mlx_destroy": (None, [_P]),
    "rs_mlx_input": (C.c_int, [_P, C.c_int, C.c_void_p, _I32P, _SZ, _ERR, _SZ]),
    "rs_mlx_op": (C.c_int, [_P, C.c_int, _U32P, _SZ, C.c_int, C.c_float, _ERR, _SZ]),
    "rs_mlx_finish": (C.c_int, [_P, C.c_uint32, C.c_void_p, _SZ, _ERR, _SZ]),
    "rs_mlx_kernel": (C.c_int, [_P, C.c_int, _U32P, _SZ, _I32P, _SZ, _F32P, _SZ, _ERR, _SZ]),
    "rs_mlx_parameter": (C.c_int, [_P, _P, C.c_char_p, _I32P, _SZ, C.c_int, _ERR, _SZ]),
    "rs_mlx_cleanup": (None, []),
    "rs_qwen_device_create": (_P, [_P, C.c_int, C.POINTER(RsQwenConfig), C.POINTER(RsQwenLayer), _SZ, _SZ,
                                   C.c_uint64, _ERR, _SZ]),
    "rs_qwen_device_destroy": (None, [_P]),
    "rs_qwen_device_decode_batch": (C.c_int, [_P, _SIDP, _U32P, _SZ, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_step": (C.c_int, [_P, _SIDP, _SZ, _U32P, _SZ, _SIDP, _F32P, _SZ, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_step_sampled": (C.c_int, [_P, _SIDP, _SZ, _U32P, _SZ, _SIDP, _U32P, _ERR, _SZ]),
    "rs_qwen_device_block": (C.c_int, [_P, _SIDP, _SZ, _U32P, _SZ, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_hidden_step": (C.c_int, [_P, _SIDP, _SZ, _U32P, _SZ, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_hidden_block": (C.c_int, [_P, _SIDP, _SZ, _U32P, _SZ, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_hidden_snapshot": (C.c_int, [_P, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_release": (C.c_int, [_P, _SIDP, _ERR, _SZ]),
    "rs_qwen_device_snapshot": (C.c_int, [_P, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_stats": (C.c_int, [_P, C.POINTER(C.c_uint64), _SZ, _ERR, _SZ]),
    "rs_qwen_device_drain": (C.c_int, [_P, C.POINTER(C.c_uint64), _ERR, _SZ]),
    "rs_qwen_device_mtp_attach": (C.c_int, [_P, _P, _ERR, _SZ]),
    "rs_qwen_device_mtp_step": (C.c_int, [_P, _SIDP, _SIDP, C.c_int, _SZ, _U32P, _SZ, _SIDP, _F32P, _SZ,
                                          C.c_int, _ERR, _SZ]),
    "rs_qwen_device_mtp_release": (C.c_int, [_P, _SIDP, _ERR, _SZ]),
    "rs_qwen_device_mtp_snapshot": (C.c_int, [_P, _SIDP, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_step_ragged": (C.c_int, [_P, _SZ, _SIDP, _U32P, _U32P, _U32P, C.c_uint32, _SIDP, _U32P, _SZ,
                                             _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_step_ragged_choices": (C.c_int, [_P, _SZ, _SIDP, _U32P, _U32P, _U32P, C.c_uint32, _U32P, _U32P,
                                                     _SZ, _SIDP, _U32P, _SZ, _F32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_mtp_verify_accept": (C.c_int, [_P, _SZ, _SIDP, _U32P, _U32P, _U32P, _SZ, _U32P, _SZ,
                                                   C.c_uint32, _SIDP, _U32P, _U32P, _U32P, _ERR, _SZ]),
    "rs_qwen_device_synthetic_state": (C.c_int, [_P, _SZ, C.c_uint64, _SIDP, _ERR, _SZ]),
    "rs_qwen_device_set_capture": (C.c_int, [_P, C.c_int, _ERR, _SZ]),
    "rs_qwen_device_set_profile": (C.c_int, [_P, C.c_int, _ERR, _SZ]),
    "rs_qwen_ep_unique_id": (C.c_int, [C.c_void_p, _SZ, _ERR, _SZ]),
    "rs_qwen_device_ep_init": (C.c_int, [_P, C.c_int, C.c_int, C.c_void_p, _SZ, _SZ, _ERR, _SZ]),
    "rs_qwen_device_ep_window": (C.c_int, [_P, C.c_int, C.c_int, _SZ, C.c_void_p, _SZ, _ERR, _SZ]),
    "rs_qwen_device_ep_connect": (C.c_int, [_P, C.c_void_p, _SZ, _ERR, _SZ]),
    "rs_qwen_device_timing": (C.c_int, [_P, C.POINTER(C.c_double), _SZ, _ERR, _SZ]),
    "rs_qwen_device_debug_routing": (C.c_int, [_P, _I32P, _SZ, _ERR, _SZ]),
    "rs_qwen_device_debug_capture": (C.c_int, [_P, C.c_int, C.c_void_p, _SZ, C.POINTER(_SZ), _ERR, _SZ]),
    "rs_qwen_debug_gemm": (C.c_int, [_P, C.c_int, C.c_int, C.POINTER(C.c_uint16), _SZ, _F32P, _SZ, C.c_int,
                                     C.POINTER(C.c_double), _ERR, _SZ]),
    "rs_qwen_project_noalloc": (C.c_int, [_P, C.c_int, C.c_int, C.c_void_p, _SZ, C.c_void_p, _SZ, C.c_void_p,
                                          _ERR, _SZ]),
}

_lib = None


def load(path: Path | None = None):
    """Load libqwen_b200.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise FileNotFoundError(f"{p} missing: build it with python {PKG / 'build.py'}")
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _errbuf():
    return C.create_string_buffer(1024)


def _call(name, *args):
    e = _errbuf()
    rc = getattr(load(), name)(*args, e, len(e))
    if rc != 0:
        raise NativeError(f"{name}: {e.value.decode(errors='replace')}")


def _ptr(a, t):
    return None if a is None else a.ctypes.data_as(C.POINTER(t))


def config(**kw) -> RsQwenConfig:
    c = RsQwenConfig()
    defaults = dict(activation_precision=1, layer_group=1, validation_mode=0, validation_interval=1,
                    chunk=8, group=64, bits=4, epsilon=1e-6, theta=1e7, interval=4, conv=4)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(c, k, v)
    return c


def config0(context: int = 512) -> RsQwenConfig:
    """BASELINE configs[0] geometry (tiny hybrid decoder)."""
    return config(hidden=256, layers=4, vocab=4096, q_heads=4, kv_heads=1, head_dim=64, key_heads=2,
                  value_heads=4, key_dim=64, value_dim=64, experts=16, top=2, intermediate=128, shared=128,
                  context=context, rope_dims=16)


def config1(layers: int = 48, context: int = 32768 + 64, vocab: int = 151936) -> RsQwenConfig:
    """BASELINE configs[1] geometry: Qwen3-Next-80B-A3B shapes."""
    return config(hidden=2048, layers=layers, vocab=vocab, q_heads=16, kv_heads=2, head_dim=256, key_heads=16,
                  value_heads=32, key_dim=128, value_dim=128, experts=512, top=10, intermediate=512, shared=512,
                  context=context, rope_dims=64)


def layer_program(cfg: RsQwenConfig):
    arr = (RsQwenLayer * cfg.layers)()
    for i in range(cfg.layers):
        arr[i].index = i
        arr[i].mixer = int((i + 1) % cfg.interval == 0)
    return arr


def state_count(cfg: RsQwenConfig) -> int:
    return load().rs_qwen_state_count(C.byref(cfg))


def ep_unique_id() -> bytes:
    """NCCL unique id (128 bytes) for rs_qwen_device_ep_init, made by rank 0."""
    buf = (C.c_uint8 * 128)()
    _call("rs_qwen_ep_unique_id", buf, 128)
    return bytes(buf)


class WeightStore:
    def __init__(self):
        e = _errbuf()
        self.h = load().rs_mlx_weights_create(e, len(e))
        if not self.h:
            raise NativeError(e.value.decode())

    def synthetic(self, cfg: RsQwenConfig, seed: int, mtp: bool = False):
        self.cfg = cfg
        _call("rs_qwen_weights_synthetic", self.h, C.byref(cfg), seed, int(mtp))
        return self

    def load(self, path):
        """Read one safetensors shard (rs_mlx_weights_load); the device layout is
        built when the first session is created on the store."""
        _call("rs_mlx_weights_load", self.h, str(path).encode())
        return self

    def quant(self, module: str, group: int, bits: int):
        """Per-module quantization override (rs_qwen_quant)."""
        _call("rs_qwen_quant", self.h, module.encode(), group, bits)
        return self

    def forward(self, cfg: RsQwenConfig, tokens, offset: int, old_state=None):
        """rs_qwen_forward: returns (last-row logits [vocab], new_state [state_count])."""
        tok = np.ascontiguousarray(tokens, np.uint32)
        n = state_count(cfg)
        new = np.zeros(n, np.float32)
        old = None if old_state is None else np.ascontiguousarray(old_state, np.float32)
        logits = np.zeros(cfg.vocab, np.float32)
        layers = layer_program(cfg)
        _call("rs_qwen_forward", self.h, 1, C.byref(cfg), layers, cfg.layers, _ptr(tok, C.c_uint32), len(tok),
              offset, _ptr(old, C.c_float), 0 if old is None else old.size, _ptr(new, C.c_float), n,
              _ptr(logits, C.c_float), logits.size, 0, None, 0, None, 0)
        return logits, new

    def weight_bytes(self, name: str, offset: int, count: int, dtype: int = 2) -> bytes:
        buf = (C.c_uint8 * count)()
        _call("rs_mlx_weight_bytes", self.h, name.encode(), None, 0, dtype, offset, buf, count)
        return bytes(buf)

    def close(self):
        if getattr(self, "h", None):
            load().rs_mlx_weights_destroy(self.h)
            self.h = None

    __del__ = close


class DeviceSession:
    """Mirror of QwenDeviceExecutor's native session (src/serving/native_device.rs)."""

    def __init__(self, store: WeightStore, cfg: RsQwenConfig, slots: int, budget_bytes: int):
        self.store, self.cfg = store, cfg
        self.layers = layer_program(cfg)
        e = _errbuf()
        self.h = load().rs_qwen_device_create(store.h, 1, C.byref(cfg), self.layers, cfg.layers, slots,
                                              budget_bytes, e, len(e))
        if not self.h:
            raise NativeError(f"rs_qwen_device_create: {e.value.decode()}")

    def close(self):
        if getattr(self, "h", None):
            load().rs_qwen_device_destroy(self.h)
            self.h = None

    __del__ = close

    def step_ragged(self, parents, positions, counts, tokens, flags=RAGGED_SAMPLED, logits_out=None,
                    sampled_out=None):
        """parents: list of StateId or None. Returns (outs, sampled, logits)."""
        n = len(positions)
        par = (StateId * n)()
        for i, p in enumerate(parents):
            if p is not None:
                par[i] = p
        pos = np.ascontiguousarray(positions, np.uint32)
        cnt = np.ascontiguousarray(counts, np.uint32)
        tok = np.ascontiguousarray(tokens, np.uint32)
        rows = int(cnt.sum()) if flags & RAGGED_ALL_ROWS else n
        outs = (StateId * n)()
        sampled = None
        if flags & RAGGED_SAMPLED:
            sampled = sampled_out if sampled_out is not None else np.zeros(rows, np.uint32)
        logits = None
        if flags & RAGGED_LOGITS:
            logits = logits_out if logits_out is not None else np.zeros((rows, self.cfg.vocab), np.float32)
        _call("rs_qwen_device_step_ragged", self.h, n, par, _ptr(pos, C.c_uint32), _ptr(cnt, C.c_uint32),
              _ptr(tok, C.c_uint32), flags, outs, _ptr(sampled, C.c_uint32), 0 if sampled is None else rows,
              _ptr(logits, C.c_float), 0 if logits is None else logits.size)
        return list(outs), sampled, logits

    def step_ragged_choices(self, parents, positions, counts, tokens, allowed, flags=RAGGED_SAMPLED):
        """step_ragged with constrained greedy selection: allowed[r] is the list of
        legal ids of output row r (empty / None = unconstrained).
        Returns (outs, sampled, logits or None)."""
        n = len(positions)
        par = (StateId * n)()
        for i, p in enumerate(parents):
            if p is not None:
                par[i] = p
        pos = np.ascontiguousarray(positions, np.uint32)
        cnt = np.ascontiguousarray(counts, np.uint32)
        tok = np.ascontiguousarray(tokens, np.uint32)
        rows = int(cnt.sum()) if flags & RAGGED_ALL_ROWS else n
        if len(allowed) != rows:
            raise ValueError("one allowed list per output row")
        lens = [0 if a is None else len(a) for a in allowed]
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
        ids = np.concatenate([np.asarray(a, np.uint32) for a in allowed if a is not None and len(a)] or
                             [np.zeros(0, np.uint32)]).astype(np.uint32)
        outs = (StateId * n)()
        sampled = np.zeros(rows, np.uint32)
        logits = np.zeros((rows, self.cfg.vocab), np.float32) if flags & RAGGED_LOGITS else None
        _call("rs_qwen_device_step_ragged_choices", self.h, n, par, _ptr(pos, C.c_uint32), _ptr(cnt, C.c_uint32),
              _ptr(tok, C.c_uint32), flags | RAGGED_SAMPLED, _ptr(offs, C.c_uint32),
              _ptr(ids, C.c_uint32) if ids.size else None, ids.size, outs, _ptr(sampled, C.c_uint32), rows,
              _ptr(logits, C.c_float), 0 if logits is None else logits.size)
        return list(outs), sampled, logits

    def decode_batch(self, parents, tokens):
        n = len(parents)
        par = (StateId * n)(*parents)
        tok = np.ascontiguousarray(tokens, np.uint32)
        outs = (StateId * n)()
        logits = np.zeros((n, self.cfg.vocab), np.float32)
        _call("rs_qwen_device_decode_batch", self.h, par, _ptr(tok, C.c_uint32), n, outs,
              _ptr(logits, C.c_float), logits.size)
        return list(outs), logits

    def step(self, previous, position, tokens, block=False, hidden=False):
        tok = np.ascontiguousarray(tokens, np.uint32)
        out = StateId()
        rows = len(tok) if block else 1
        logits = np.zeros((rows, self.cfg.vocab), np.float32)
        prev = C.byref(previous) if previous is not None else None
        name = {(False, False): "rs_qwen_device_step", (True, False): "rs_qwen_device_block",
                (False, True): "rs_qwen_device_hidden_step", (True, True): "rs_qwen_device_hidden_block"}[(block, hidden)]
        if name == "rs_qwen_device_step":
            _call(name, self.h, prev, position, _ptr(tok, C.c_uint32), len(tok), C.byref(out),
                  _ptr(logits, C.c_float), logits.size, None, 0)
        else:
            _call(name, self.h, prev, position, _ptr(tok, C.c_uint32), len(tok), C.byref(out),
                  _ptr(logits, C.c_float), logits.size)
        return out, logits

    def step_sampled(self, previous, position, tokens):
        tok = np.ascontiguousarray(tokens, np.uint32)
        out, token = StateId(), C.c_uint32()
        prev = C.byref(previous) if previous is not None else None
        _call("rs_qwen_device_step_sampled", self.h, prev, position, _ptr(tok, C.c_uint32), len(tok),
              C.byref(out), C.byref(token))
        return out, token.value

    def release(self, sid: StateId):
        _call("rs_qwen_device_release", self.h, C.byref(sid))

    def verify_accept(self, parents, seeds, drafts, eos=(), flags=0, width=None):
        """Speculative verify + accept (rs_qwen_device_mtp_verify_accept).
        drafts: list of per-sequence draft lists. Returns (outs, accepted, emitted lists)."""
        n = len(parents)
        width = max([len(x) for x in drafts] + [0]) if width is None else width
        par = (StateId * n)(*parents)
        seed = np.ascontiguousarray(seeds, np.uint32)
        nd = np.array([len(x) for x in drafts], np.uint32)
        dr = np.zeros((n, max(width, 1)), np.uint32)
        for i, x in enumerate(drafts):
            dr[i, :len(x)] = x
        eo = np.ascontiguousarray(eos, np.uint32)
        outs = (StateId * n)()
        acc = np.zeros(n, np.uint32)
        em = np.zeros((n, width + 1), np.uint32)
        ne = np.zeros(n, np.uint32)
        _call("rs_qwen_device_mtp_verify_accept", self.h, n, par, _ptr(seed, C.c_uint32), _ptr(dr, C.c_uint32),
              _ptr(nd, C.c_uint32), width, _ptr(eo, C.c_uint32) if len(eo) else None, len(eo), flags, outs,
              _ptr(acc, C.c_uint32), _ptr(em, C.c_uint32), _ptr(ne, C.c_uint32))
        return list(outs), [int(a) for a in acc], [list(map(int, em[i, :ne[i]])) for i in range(n)]

    def snapshot(self, sid: StateId):
        n = state_count(self.cfg)
        out = np.zeros(n, np.float32)
        _call("rs_qwen_device_snapshot", self.h, C.byref(sid), _ptr(out, C.c_float), n)
        return out

    def hidden_snapshot(self, sid: StateId, rows: int):
        out = np.zeros((rows, self.cfg.hidden), np.float32)
        _call("rs_qwen_device_hidden_snapshot", self.h, C.byref(sid), _ptr(out, C.c_float), out.size)
        return out

    def stats(self):
        out = (C.c_uint64 * STATS_COUNT)()
        _call("rs_qwen_device_stats", self.h, out, STATS_COUNT)
        return list(out)

    def drain(self) -> int:
        n = C.c_uint64()
        _call("rs_qwen_device_drain", self.h, C.byref(n))
        return n.value

    def mtp_attach(self, store):
        _call("rs_qwen_device_mtp_attach", self.h, store.h)

    def mtp_step(self, previous, source, tokens, row: int = 0, draft_source: int = 0):
        """One MTP draft step (rs_qwen_device_mtp_step); returns (draft version, last-row logits)."""
        tok = np.ascontiguousarray(tokens, np.uint32)
        out = StateId()
        logits = np.zeros(self.cfg.vocab, np.float32)
        _call("rs_qwen_device_mtp_step", self.h, None if previous is None else C.byref(previous), C.byref(source),
              draft_source, row, _ptr(tok, C.c_uint32), len(tok), C.byref(out), _ptr(logits, C.c_float),
              logits.size, 0)
        return out, logits

    def mtp_release(self, sid: StateId):
        _call("rs_qwen_device_mtp_release", self.h, C.byref(sid))

    def mtp_snapshot(self, sid: StateId, rows: int):
        """(K [kv, context, d], V [kv, context, d], hidden [rows, hidden]) of a draft version."""
        c = self.cfg
        per = c.kv_heads * c.context * c.head_dim
        out = np.zeros(2 * per + rows * c.hidden, np.float32)
        _call("rs_qwen_device_mtp_snapshot", self.h, C.byref(sid), _ptr(out, C.c_float), out.size)
        kv = out[:2 * per].reshape(2, c.kv_heads, c.context, c.head_dim)
        return kv[0], kv[1], out[2 * per:].reshape(rows, c.hidden)

    def synthetic_state(self, position: int, seed: int) -> StateId:
        out = StateId()
        _call("rs_qwen_device_synthetic_state", self.h, position, seed, C.byref(out))
        return out

    def set_capture(self, routing: bool):
        _call("rs_qwen_device_set_capture", self.h, int(routing))

    def ep_init(self, world: int, rank: int, uid: bytes, cap_tokens: int):
        """Join the expert-parallel group (see rs_qwen_device_ep_init)."""
        buf = (C.c_uint8 * len(uid)).from_buffer_copy(uid)
        _call("rs_qwen_device_ep_init", self.h, world, rank, buf, len(uid), cap_tokens)

    def ep_window(self, world: int, rank: int, cap_tokens: int) -> bytes:
        """Expert parallelism over direct NVLink stores, step 1: allocate this
        rank's window; returns its CUDA IPC handle (64 bytes) for the peers."""
        buf = (C.c_uint8 * 64)()
        _call("rs_qwen_device_ep_window", self.h, world, rank, cap_tokens, buf, 64)
        return bytes(buf)

    def ep_connect(self, handles):
        """Step 2: every rank's window handle, in rank order."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _call("rs_qwen_device_ep_connect", self.h, buf, len(blob))

    def set_profile(self, on: bool):
        _call("rs_qwen_device_set_profile", self.h, int(on))

    def timing(self):
        """(last step device ms, cumulative device ms, timed steps, per-stage ms[19])."""
        out = (C.c_double * 22)()
        _call("rs_qwen_device_timing", self.h, out, 22)
        return out[0], out[1], int(out[2]), list(out[3:])

    def debug_gemm(self, which: int, layer: int, x_f16, rows: int, engine: int = 0):
        """Run one dense GEMM (0 in_proj, 1 out_proj, 2 router, 3 lm_head) on IEEE-half
        input bits [T][k]; returns (y, ms)."""
        x = np.ascontiguousarray(x_f16, np.uint16)
        T = x.shape[0]
        y = np.zeros((T, rows), np.float32)
        ms = C.c_double()
        _call("rs_qwen_debug_gemm", self.h, which, layer, x.ctypes.data_as(C.POINTER(C.c_uint16)), T,
              _ptr(y, C.c_float), y.size, engine, C.byref(ms))
        return y, ms.value

    def project_noalloc(self, which: int, layer: int, x_device_ptr: int, T: int, y_device_ptr: int, y_count: int,
                        stream_ptr: int = 0):
        """Allocation-free dense projection on device buffers (rs_qwen_project_noalloc):
        y (fp32 [T][rows]) = x (IEEE half [T][k]) . W; raises on error, including T x rows
        beyond the 16 MiB static scratch."""
        _call("rs_qwen_project_noalloc", self.h, which, layer, C.c_void_p(x_device_ptr), T,
              C.c_void_p(y_device_ptr), y_count, C.c_void_p(stream_ptr or None))

    def debug_capture(self, what: int, dtype=np.int32, capacity: int = 1 << 26):
        """Raw last-step intermediates (see rs_qwen_device_debug_capture)."""
        buf = np.zeros(capacity // np.dtype(dtype).itemsize, dtype)
        n = C.c_size_t()
        _call("rs_qwen_device_debug_capture", self.h, what, buf.ctypes.data_as(C.c_void_p), buf.nbytes, C.byref(n))
        return buf[: n.value // np.dtype(dtype).itemsize].copy()

    def debug_routing(self, tokens: int):
        out = np.zeros((self.cfg.layers, tokens, self.cfg.top), np.int32)
        _call("rs_qwen_device_debug_routing", self.h, _ptr(out, C.c_int32), out.size)
        return out
