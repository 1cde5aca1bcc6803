"""The C-ABI library loads and exports every symbol include/*.h declares
(no compute call: this runs without a GPU)."""
import ctypes as C
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[\w\s\*]+?\b(rs_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_reference_surface():
    names = declared_symbols()
    # the reference's device ABI (native/mlx_bridge.h:76-115) must all be present
    for sym in ("rs_qwen_device_create", "rs_qwen_device_decode_batch", "rs_qwen_device_step",
                "rs_qwen_device_step_sampled", "rs_qwen_device_block", "rs_qwen_device_release",
                "rs_qwen_device_snapshot", "rs_qwen_device_stats", "rs_qwen_device_drain",
                "rs_qwen_device_destroy", "rs_qwen_device_hidden_step", "rs_qwen_device_hidden_block",
                "rs_qwen_device_hidden_snapshot", "rs_qwen_device_mtp_attach", "rs_qwen_device_mtp_step",
                "rs_qwen_device_mtp_release", "rs_qwen_device_mtp_snapshot", "rs_qwen_quant",
                "rs_mlx_weights_create", "rs_mlx_weights_destroy", "rs_mlx_weights_load",
                "rs_mlx_weight_bytes", "rs_mlx_version"):
        assert sym in names, sym


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load()
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, missing
    # every declared symbol also has a ctypes signature in the host binding
    assert set(pkg.SIGNATURES) >= declared_symbols()


def test_struct_layouts(pkg):
    assert C.sizeof(pkg.RsQwenConfig) == 132  # native/mlx_bridge.h:50-53
    assert C.sizeof(pkg.StateId) == 40        # native/state_table.h:13
    assert C.sizeof(pkg.RsQwenLayer) == 8


def test_state_count_matches_oracle(pkg, O):
    for cfg_p, cfg_o in ((pkg.config0(), O.config0()), (pkg.config1(layers=8, context=4096), O.config1(layers=8, context=4096))):
        assert pkg.state_count(cfg_p) == O.lib().orc_state_count(C.byref(cfg_o))


def test_library_exports_every_symbol_the_rust_crate_links(pkg):
    """Every `extern "C"` name the reference's Rust crate declares (committed
    list, tests/golden/make_ffi_list.py) is declared in include/*.h and
    exported by the library, so the crate links unchanged."""
    wanted = (ROOT / "tests" / "golden" / "rust_ffi_symbols.txt").read_text().split()
    assert len(wanted) == 32
    lib = pkg.load()
    declared = declared_symbols()
    assert [s for s in wanted if s not in declared] == []
    assert [s for s in wanted if not hasattr(lib, s)] == []


def test_graph_builder_stubs_report_without_a_gpu(pkg):
    """The MLX graph builder has no counterpart here: the stubs answer with the
    ABI's error convention and touch no device."""
    lib = pkg.load()
    err = C.create_string_buffer(256)
    assert lib.rs_mlx_create(1, err, 256) is None
    assert b"MLX graph" in err.value
    err = C.create_string_buffer(256)
    assert lib.rs_mlx_op(None, 0, None, 0, 0, 0.0, err, 256) == -1 and err.value
    lib.rs_mlx_cleanup()
    lib.rs_mlx_destroy(None)
    err = C.create_string_buffer(256)
    assert lib.rs_qwen_forward(None, 1, None, None, 0, None, 0, 0, None, 0, None, 0, None, 0, 0, None, 0, None, 0,
                               err, 256) == -1
    assert b"descriptor" in err.value
