"""Host-side checks that need no GPU: the C ABI loads and exports every
declared symbol, the pure-host queries agree with the oracle, and the
product's config/module tree matches the reference's."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from oracle import parrot_oracle as po
from parrot_b200 import ModelConfig, Parrot, _lib
from parrot_b200 import build as pbuild

HEADER = Path(__file__).resolve().parent.parent / "include" / "parrot_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(parrot_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    pbuild.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_names()) == names


def _header_prototypes() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, parameter declarations) of every prototype in the header."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(parrot_\w+)\s*\(([^;{]*?)\)\s*;", text,
                         flags=re.S):
        params = m.group(3).strip()
        protos[m.group(2)] = (" ".join(m.group(1).split()),
                              [] if params in ("", "void") else [q.strip() for q in params.split(",")])
    return protos


def _expected_ctype(decl: str):
    """The ctypes type a C declaration (type and name) must be bound as, or
    "pointer" for any pointer (bound as c_void_p, c_char_p or POINTER(...))."""
    if "*" in decl:
        return "pointer"
    t = " ".join(decl.replace("const", "").split()[:-1])
    return {"int": ctypes.c_int, "float": ctypes.c_float, "size_t": ctypes.c_size_t,
            "long long": ctypes.c_longlong, "int64_t": ctypes.c_int64,
            "unsigned long long": ctypes.c_ulonglong}[t]


def _matches(ct, want) -> bool:
    if want == "pointer":
        return ct in (ctypes.c_void_p, ctypes.c_char_p) or (
            isinstance(ct, type) and issubclass(ct, ctypes._Pointer))
    return ct is want


def test_ctypes_signatures_match_the_header():
    """Every entry point's ctypes binding has the header's parameter count,
    parameter types and return type, so a prototype changed on one side only
    fails here rather than on a GPU."""
    protos = _header_prototypes()
    assert sorted(protos) == sorted(_lib._SIGNATURES)
    for name, (res, args) in _lib._SIGNATURES.items():
        ret, params = protos[name]
        assert len(args) == len(params), name
        for i, (decl, ct) in enumerate(zip(params, args)):
            assert _matches(ct, _expected_ctype(decl)), (name, i, decl, ct)
        assert _matches(res, _expected_ctype(ret + " r")), (name, ret, res)


def test_version_and_error_string(lib):
    assert lib.parrot_b200_version() == 100
    assert isinstance(lib.parrot_b200_last_error(), bytes)


@pytest.mark.parametrize("tokens,experts", [(0, 16), (1, 16), (256, 16), (512, 16), (16384, 16),
                                            (7, 4), (33, 2), (100, 32)])
def test_capacity_matches_oracle(lib, tokens, experts):
    assert lib.parrot_moe_capacity(tokens, experts) == po.expert_capacity(2 * tokens, experts)


def test_workspace_layout_is_aligned_and_ordered(lib):
    dims = _lib.MoeDims(512, 768, 16, 2, 512, 256, 0)
    lay = _lib.MoeLayout()
    assert lib.parrot_moe_workspace_layout(ctypes.byref(dims), ctypes.byref(lay)) == 0
    offsets = [getattr(lay, n) for n in _lib.LAYOUT_OFFSETS]
    assert all(o % 256 == 0 for o in offsets)
    assert lay.capacity == 128
    assert lay.grouped_rows == 16 * 128 + 1024
    assert lay.route_blocks == 128  # 4-token router tiles up to T = 4096
    assert lay.shared_y + 512 * 768 * 2 <= lay.total


def test_slot_mode_layout(lib):
    """capacity -2 (slot mode): a 2T-row region per expert, no overflow region
    needed; the status region grows by the E expert counters and a ticket."""
    plain, slots = _lib.MoeLayout(), _lib.MoeLayout()
    assert lib.parrot_moe_workspace_layout(
        ctypes.byref(_lib.MoeDims(512, 768, 16, 2, 512, 256, 0)), ctypes.byref(plain)) == 0
    assert lib.parrot_moe_workspace_layout(
        ctypes.byref(_lib.MoeDims(512, 768, 16, 2, 512, 256, -2)), ctypes.byref(slots)) == 0
    assert slots.capacity == 1024
    assert slots.grouped_rows == 16 * 1024 + 1024
    assert slots.status == 0 and slots.indices >= 16 + 4 * (16 + 1)
    assert slots.indices == plain.indices
    bad = _lib.MoeDims(512, 768, 16, 2, 512, 256, -3)
    assert lib.parrot_moe_workspace_layout(ctypes.byref(bad), ctypes.byref(slots)) == \
        _lib.PARROT_EINVAL


@pytest.mark.parametrize("field,value", [("top_k", 1), ("dim", 96), ("n_experts", 33),
                                         ("expert_dim", 100), ("shared_dim", 0)])
def test_layout_rejects_unsupported_dims(lib, field, value):
    d = dict(tokens=8, dim=768, n_experts=16, top_k=2, expert_dim=512, shared_dim=256, capacity=0)
    d[field] = value
    dims = _lib.MoeDims(**d)
    lay = _lib.MoeLayout()
    assert lib.parrot_moe_workspace_layout(ctypes.byref(dims), ctypes.byref(lay)) == _lib.PARROT_EINVAL
    assert lib.parrot_b200_last_error()


def test_entry_points_reject_bad_arguments_before_launch(lib):
    # argument errors are detected on the host, so these need no GPU
    assert lib.parrot_rmsnorm_bf16(None, None, None, 4, 100, 1e-6, None) == _lib.PARROT_EINVAL
    assert lib.parrot_depthmix_bf16(None, None, 0, None, None, 1e-6, None, 1e-6, None, None,
                                    None, None, 4, 768, None) == _lib.PARROT_EINVAL
    assert lib.parrot_pack_gate_up_bf16(None, None, None, 1, 100, 768, None) == _lib.PARROT_EINVAL
    dims = _lib.MoeDims(4, 768, 16, 2, 512, 256, 0)
    w = _lib.MoeWeights()
    o = _lib.MoeOutputs()
    assert lib.parrot_moe_forward_bf16(ctypes.byref(dims), ctypes.byref(w), None, ctypes.byref(o),
                                       None, 0, None) == _lib.PARROT_EINVAL


def test_decode_entry_points_reject_bad_arguments_before_launch(lib):
    E = _lib.PARROT_EINVAL
    # small-batch projections: at most 8 rows, n_out % 16, k_in % 8 and <= 1024, pointers
    assert lib.parrot_linear_small(None, 0, None, 0, None, 0, 9, 768, 768, None) == E
    assert lib.parrot_linear_small(None, 0, None, 0, None, 0, 1, 100, 768, None) == E
    assert lib.parrot_linear_small(None, 0, None, 0, None, 0, 1, 768, 2048, None) == E
    assert lib.parrot_linear_small(None, 0, None, 0, None, 0, 1, 768, 768, None) == E
    assert lib.parrot_linear_small(None, 0, None, 0, None, 0, 0, 768, 768, None) == _lib.PARROT_OK
    # RoPE inside decode attention: tables must cover every cache position
    assert lib.parrot_decode_attention_rope_bf16(
        None, 0, None, 0, None, None, 0, None, None, None, 1, 8, 2, 4096, 96, 2048, 0.1,
        None, None, 4096, None, 0, None, None) == E
    assert lib.parrot_decode_attention_rope_bf16(
        None, 0, None, 0, None, None, 0, None, None, None, 1, 8, 2, 4096, 96, 2048, 0.1,
        ctypes.c_void_p(16), ctypes.c_void_p(16), 2048, None, 0, None, None) == E


@pytest.mark.parametrize("batch,heads,positions,dim", [(1, 8, 4096, 96), (8, 8, 4096, 128),
                                                       (64, 8, 4096, 96), (3, 4, 100, 32)])
def test_decode_attention_scratch_size(lib, batch, heads, positions, dim):
    """Partials [B, H, slots, D + 2] fp32 plus one arrival counter per (row,
    head); slots = min(32-key chunks, max(1, 256 // B))."""
    chunks = (positions + 31) // 32
    slots = min(chunks, max(1, 256 // batch))
    want = batch * heads * slots * (dim + 2) * 4 + batch * heads * 4
    assert lib.parrot_decode_attention_scratch_bytes(batch, heads, positions, dim) == want


def tiny_b200(**kw):
    base = dict(vocab_size=32768, dim=128, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=32,
                kv_latent_dim=32, n_experts=8, expert_dim=128, shared_expert_dim=64,
                window_size=128, max_seq_len=512)
    base.update(kw)
    return ModelConfig(**base)


def test_seeded_init_and_state_dict_match_reference_layout():
    torch.manual_seed(0)
    model = Parrot(tiny_b200())
    torch.manual_seed(0)
    oracle = po.OracleParrot(po.tiny_config())
    a, b = model.state_dict(), oracle.state_dict()
    assert list(a) == list(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_default_config_is_parrot_xl():
    cfg = ModelConfig()
    assert (cfg.dim, cfg.n_layers, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim) == \
        (768, 16, 16, 512, 256)
    assert cfg.depth_sources == 9


@pytest.mark.parametrize("kw,msg", [
    (dict(moe_backend="pytorch"), "moe_backend"),
    (dict(depth_backend="metal"), "depth_backend"),
    (dict(top_k=1), "top_k"),
    (dict(n_experts=33), "experts"),
    (dict(dim=96, n_heads=1, n_kv_heads=1), "dim"),
    (dict(expert_dim=500), "expert widths"),
    (dict(n_heads=3), "n_heads"),
    (dict(norm_eps=0.0), "norm_eps"),
    (dict(vocab_size=0), "vocab_size"),
])
def test_config_validation(kw, msg):
    with pytest.raises(ValueError, match=msg):
        ModelConfig(**kw)


def test_parameter_counts_match_reference_formula():
    cfg = tiny_b200()
    torch.manual_seed(0)
    counts = Parrot(cfg).parameter_counts()
    torch.manual_seed(0)
    o = po.OracleParrot(po.tiny_config())
    total = sum(p.numel() for p in o.parameters())
    assert counts["total"] == total
    assert counts["active_per_token"] == total - cfg.n_layers * (cfg.n_experts - 2) * 3 * \
        cfg.dim * cfg.expert_dim


def test_bridge_refuses_cpu_tensors():
    from parrot_b200 import bridge
    cfg = tiny_b200()
    norm = Parrot(cfg).final_norm
    with torch.inference_mode(), pytest.raises(RuntimeError, match="CUDA"):
        bridge.b200_rms_norm(norm, torch.zeros(2, 128, dtype=torch.bfloat16))


def _ep_dims(**kw):
    d = dict(ranks=4, rank=1, max_tokens=2048, dim=768, n_experts=16, expert_dim=512, wait_ns=0)
    d.update(kw)
    return _lib.EpDims(*d.values())


def test_ep_buffer_layout_is_aligned_and_sized(lib):
    lay = _lib.EpLayout()
    assert lib.parrot_ep_buffer_layout(ctypes.byref(_ep_dims()), ctypes.byref(lay)) == 0
    offsets = [getattr(lay, n) for n in _lib.EP_LAYOUT_OFFSETS]
    assert all(o % 256 == 0 for o in offsets)
    assert offsets == sorted(offsets)
    assert lay.region_rows == 4096
    # peer-written regions: one receive region per source, one return region
    assert lay.back_rows - lay.recv_rows >= 4 * 4096 * 768 * 2
    assert lay.hidden - lay.back_rows >= 4096 * 768 * 2
    assert lay.total - lay.y >= 4 * 4096 * 768 * 2


@pytest.mark.parametrize("field,value", [("ranks", 0), ("ranks", 9), ("rank", 4), ("rank", -1),
                                         ("n_experts", 18), ("dim", 96), ("expert_dim", 100),
                                         ("max_tokens", 0)])
def test_ep_layout_rejects_unsupported_dims(lib, field, value):
    lay = _lib.EpLayout()
    assert lib.parrot_ep_buffer_layout(ctypes.byref(_ep_dims(**{field: value})),
                                       ctypes.byref(lay)) == _lib.PARROT_EINVAL
    assert b"ep:" in lib.parrot_b200_last_error()


def test_ep_calls_reject_bad_arguments_before_any_launch(lib):
    """Argument errors come back as PARROT_EINVAL without touching a device."""
    ep = _ep_dims(ranks=2, rank=0, max_tokens=64)
    peers = _lib.EpPeers()  # no buffers mapped
    dims = _lib.MoeDims(64, 768, 16, 2, 512, 256, -1)
    assert lib.parrot_moe_ep_send_bf16(ctypes.byref(dims), ctypes.byref(ep), ctypes.byref(peers),
                                       None, 0, None) == _lib.PARROT_EINVAL
    assert b"mapped" in lib.parrot_b200_last_error()
    peers.buffers[0] = peers.buffers[1] = 256
    too_many = _lib.MoeDims(65, 768, 16, 2, 512, 256, -1)
    assert lib.parrot_moe_ep_send_bf16(ctypes.byref(too_many), ctypes.byref(ep),
                                       ctypes.byref(peers), None, 0, None) == _lib.PARROT_EINVAL
    assert b"max_tokens" in lib.parrot_b200_last_error()
    capacity = _lib.MoeDims(64, 768, 16, 2, 512, 256, 0)
    assert lib.parrot_moe_ep_send_bf16(ctypes.byref(capacity), ctypes.byref(ep),
                                       ctypes.byref(peers), None, 0, None) == _lib.PARROT_EINVAL
    assert lib.parrot_moe_ep_receive(ctypes.byref(ep), None, None) == _lib.PARROT_EINVAL
    assert lib.parrot_moe_ep_experts_bf16(ctypes.byref(ep), None, None, None,
                                          None) == _lib.PARROT_EINVAL
    assert lib.parrot_ipc_export(None, None, None) == _lib.PARROT_EINVAL


def test_fused_ep_calls_reject_bad_arguments_before_any_launch(lib):
    """The dispatch + send and experts + return entry points check the same
    things as the pairs they replace, before anything is launched."""
    E = _lib.PARROT_EINVAL
    ep = _ep_dims(ranks=2, rank=1, max_tokens=64)
    unmapped = _lib.EpPeers()
    dims = _lib.MoeDims(64, 768, 16, 2, 512, 256, -1)
    w = _lib.MoeWeights()
    out = _lib.MoeOutputs(None, None, None, None, None, None, None, None)

    def dispatch_send(d, peers, weights=w, x=None):
        return lib.parrot_moe_ep_dispatch_send_bf16(
            ctypes.byref(d), ctypes.byref(weights), x, ctypes.byref(out), ctypes.byref(ep),
            ctypes.byref(peers), None, 0, None)

    assert dispatch_send(dims, unmapped) == E
    assert b"mapped" in lib.parrot_b200_last_error()
    peers = _lib.EpPeers()
    peers.buffers[0] = peers.buffers[1] = 256
    assert dispatch_send(_lib.MoeDims(65, 768, 16, 2, 512, 256, -1), peers) == E
    assert b"max_tokens" in lib.parrot_b200_last_error()
    assert dispatch_send(_lib.MoeDims(64, 768, 16, 2, 512, 256, 0), peers) == E
    assert dispatch_send(_lib.MoeDims(64, 768, 8, 2, 512, 256, -1), peers) == E
    assert dispatch_send(dims, peers) == E  # no router weight
    assert b"router" in lib.parrot_b200_last_error()
    assert lib.parrot_moe_ep_experts_return_bf16(ctypes.byref(ep), ctypes.byref(unmapped),
                                                 None, None, None) == E
    assert lib.parrot_moe_ep_experts_return_bf16(ctypes.byref(ep), ctypes.byref(peers), None,
                                                 None, None) == E
    assert b"aligned weights" in lib.parrot_b200_last_error()
    assert lib.parrot_moe_ep_experts_return_bf16(ctypes.byref(ep), ctypes.byref(peers), 8, 16,
                                                 None) == E


def test_wait_selftest_rejects_bad_arguments_before_launch(lib):
    E = _lib.PARROT_EINVAL
    assert lib.parrot_selftest_wait_timeout(0, 256, None) == E
    assert lib.parrot_selftest_wait_timeout(2_000_000_000, 256, None) == E
    assert lib.parrot_selftest_wait_timeout(1_000_000, None, None) == E
    assert lib.parrot_selftest_wait_timeout(1_000_000, 8, None) == E  # not 16-byte aligned
