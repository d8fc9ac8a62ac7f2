"""The C ABI without a GPU: the library loads, exports every symbol
include/deltacore.h declares, its structs match the header's layout, and the
host-side validation (the reference's asserts, src/delta/path.rs:177-208)
returns the documented status codes before anything touches a device."""
import ctypes
import importlib
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")


def header_functions():
    text = open(os.path.join(ROOT, "include", "deltacore.h")).read()
    return re.findall(r"DC_API\s+[\w\s\*]+?\b(dc_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    declared = header_functions()
    assert set(declared) >= {"dc_chunk_fwd", "dc_step"}
    lib = ctypes.CDLL(abi.LIB_PATH)
    for name in declared:
        assert hasattr(lib, name), name
    assert set(abi.EXPORTS) >= set(declared)


def test_version_and_status_strings():
    lib = abi.lib()
    assert lib.dc_version() >= 100
    for code in range(8):
        assert abi.status_string(code)
    assert lib.dc_last_cuda_error() == 0


def test_struct_layout_matches_the_header(tmp_path):
    """ctypes offsets equal what a C compiler gives the header's structs."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = {
        "dc_chunk_args": [f for f, _ in abi.ChunkArgs._fields_],
        "dc_step_args": [f for f, _ in abi.StepArgs._fields_],
        "dc_chunk_bwd_args": [f for f, _ in abi.ChunkBwdArgs._fields_],
        "dc_out_norm_args": [f for f, _ in abi.OutNormArgs._fields_],
        "dc_qkv_prologue_args": [f for f, _ in abi.PrologueArgs._fields_],
        "dc_gate_args": [f for f, _ in abi.GateArgs._fields_],
    }
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "deltacore.h"', "int main(void) {"]
    for st, names in fields.items():
        lines.append(f'printf("{st} sizeof %zu\\n", sizeof({st}));')
        for n in names:
            lines.append(f'printf("{st} {n} %zu\\n", offsetof({st}, {n}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    want = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l}
    for st, cls in (("dc_chunk_args", abi.ChunkArgs), ("dc_step_args", abi.StepArgs),
                    ("dc_chunk_bwd_args", abi.ChunkBwdArgs), ("dc_out_norm_args", abi.OutNormArgs),
                    ("dc_qkv_prologue_args", abi.PrologueArgs), ("dc_gate_args", abi.GateArgs)):
        assert want[(st, "sizeof")] == ctypes.sizeof(cls)
        for n, _ in cls._fields_:
            assert want[(st, n)] == getattr(cls, n).offset, (st, n)


def _args(**over):
    a = abi.ChunkArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv = 2, 9, 2, 4, 6
    a.n_householder, a.erase_w, a.write_w, a.g_w, a.chunk_len = 1, 1, 1, 1, 64
    a.in_dtype = a.gate_dtype = a.out_dtype = abi.DC_F32
    a.scale = 0.5
    fake = 0x10000  # never dereferenced: validation fails or passes before any device work
    a.q, a.k, a.v, a.erase, a.write, a.g = fake, fake + 256, fake + 512, fake + 768, fake + 1024, fake + 1280
    a.state_in, a.y, a.state_out = fake + 2048, fake + 4096, fake + 8192
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize(
    "over,status",
    [
        (dict(seq=0), abi.DC_EINVAL_SHAPE),            # path.rs:179 sequence > 0
        (dict(dk=0), abi.DC_EINVAL_SHAPE),
        (dict(erase_w=3), abi.DC_EINVAL_WIDTH),        # path.rs:187-195
        (dict(write_w=4), abi.DC_EINVAL_WIDTH),
        (dict(g_w=2), abi.DC_EINVAL_WIDTH),
        (dict(chunk_len=0), abi.DC_EINVAL_ARG),        # path.rs:219 chunk_len >= 1
        (dict(n_householder=0), abi.DC_EINVAL_ARG),
        (dict(scale=float("nan")), abi.DC_EINVAL_ARG),
        (dict(in_dtype=7), abi.DC_EUNSUPPORTED_DTYPE),
        (dict(q=None), abi.DC_EINVAL_ARG),
        (dict(g=None), abi.DC_EINVAL_ARG),             # gated without a gate
        (dict(y=0x10000), abi.DC_EINVAL_ARG),          # output aliases an input
        (dict(q=0x10001), abi.DC_EINVAL_ARG),          # misaligned
        (dict(dk=512, erase_w=1), abi.DC_EUNSUPPORTED),
        (dict(n_householder=9), abi.DC_EUNSUPPORTED),
    ],
)
def test_validation_status_codes(over, status):
    a = _args(**over)
    assert abi.lib().dc_chunk_fwd(a, None) == status
    assert abi.lib().dc_chunk_kernel_choice(a) == -status


def test_empty_batch_is_a_no_op():
    assert abi.lib().dc_chunk_fwd(_args(batch=0), None) == abi.DC_OK
    assert abi.lib().dc_chunk_launches(_args(batch=0)) == 0


def test_kernel_choice_is_host_logic():
    assert abi.lib().dc_chunk_kernel_choice(_args()) == 0  # f32, dk=4: CUDA-core kernel
    a = _args(dk=128, dv=128, in_dtype=abi.DC_BF16, flags=abi.DC_FLAG_FORCE_SIMT)
    assert abi.lib().dc_chunk_kernel_choice(a) == 0


def test_fp32_chunked_path_choice_is_host_logic():
    """fp32 inputs (the reference's precision) with a workspace take the chunked tensor-core path (3): two
    launches; a short workspace is DC_EWORKSPACE; per-channel log-decays, dk > 128, FORCE_SIMT and no
    workspace stay on the CUDA-core kernel."""
    lib = abi.lib()
    need = lib.dc_chunk_workspace_size(_args())
    assert need > 0
    ws = dict(workspace=0x400000, workspace_bytes=need)
    assert lib.dc_chunk_kernel_choice(_args(**ws)) == 3
    assert lib.dc_chunk_launches(_args(**ws)) == 2
    assert lib.dc_chunk_kernel_choice(_args(workspace=0x400000, workspace_bytes=need - 1)) == -abi.DC_EWORKSPACE
    assert lib.dc_chunk_kernel_choice(_args(flags=abi.DC_FLAG_FORCE_SIMT, **ws)) == 0
    assert lib.dc_chunk_workspace_size(_args(g_w=4)) == 0  # per-channel log-decay
    assert lib.dc_chunk_kernel_choice(_args(g_w=4, **ws)) == 0
    big = _args(dk=200, dv=8, erase_w=1)
    assert lib.dc_chunk_workspace_size(big) == 0
    # bf16 at d = 128 stays on the fused kernel; bf16 at d = 64 takes the chunked path
    assert lib.dc_chunk_workspace_size(_args(dk=128, dv=128, in_dtype=abi.DC_BF16)) == 0
    assert lib.dc_chunk_workspace_size(_args(dk=64, dv=64, in_dtype=abi.DC_BF16)) > 0
    # u micro-steps fold into 32-row chunks: seq 9 x u 4 = 36 rows, two chunks
    assert lib.dc_chunk_workspace_size(_args(n_householder=4)) > need


def test_stall_hook_is_taken_by_the_tensor_core_kernel_only():
    a = _args(dk=128, dv=128, in_dtype=abi.DC_BF16, flags=abi.DC_FLAG_TEST_STALL)
    assert abi.lib().dc_chunk_kernel_choice(a) == 1
    for flags in (abi.DC_FLAG_TEST_STALL, abi.DC_FLAG_TEST_STALL | abi.DC_FLAG_RECURRENT):
        assert abi.lib().dc_chunk_kernel_choice(_args(flags=flags)) == -abi.DC_EINVAL_ARG
        assert abi.lib().dc_chunk_launches(_args(flags=flags)) == -abi.DC_EINVAL_ARG
    a = _args(dk=128, dv=128, in_dtype=abi.DC_BF16, flags=abi.DC_FLAG_TEST_STALL | abi.DC_FLAG_FORCE_SIMT)
    assert abi.lib().dc_chunk_kernel_choice(a) == -abi.DC_EINVAL_ARG


def test_step_validation():
    s = abi.StepArgs()
    s.batch, s.heads, s.dk, s.dv = 2, 2, 4, 6
    s.n_householder, s.erase_w, s.write_w, s.g_w = 1, 1, 5, 0
    s.scale = 0.5
    s.q = s.k = s.v = s.erase = s.write = 0x10000
    s.state_in = s.state_out = 0x20000
    s.y = 0x30000
    assert abi.lib().dc_step(s, None) == abi.DC_EINVAL_WIDTH


def test_python_mirror_rejects_cpu_tensors():
    import torch
    q = torch.zeros(1, 2, 1, 4)
    inp = dn.DeltaInput(q, q, torch.zeros(1, 2, 1, 6), torch.zeros(1, 2, 1, 1), torch.zeros(1, 2, 1, 1),
                        None, torch.zeros(1, 1, 4, 6))
    with pytest.raises(dn.DeltaCoreError):
        inp.run()


def test_python_mirror_sanity_mirrors_the_reference_asserts():
    import torch
    q = torch.zeros(1, 2, 1, 4)
    bad = dn.DeltaInput(q, q, torch.zeros(1, 2, 1, 6), torch.zeros(1, 2, 1, 3), torch.zeros(1, 2, 1, 1),
                        None, torch.zeros(1, 1, 4, 6))
    with pytest.raises(dn.DeltaShapeError):
        bad.sanity()
    empty = dn.DeltaInput(torch.zeros(1, 0, 1, 4), torch.zeros(1, 0, 1, 4), torch.zeros(1, 0, 1, 6),
                          torch.zeros(1, 0, 1, 1), torch.zeros(1, 0, 1, 1), None, torch.zeros(1, 1, 4, 6))
    with pytest.raises(dn.DeltaShapeError):
        empty.sanity()
    assert dn.DeltaPath.default().resolved_chunk_len() == 64
    assert dn.DeltaPath.Recurrent().resolved_chunk_len() == 1
    assert dn.DeltaPath.with_chunk_len(16).resolved_chunk_len() == 16


def test_python_mirror_nan_inf_guard_is_opt_in():
    """The reference's `san` guard (src/delta/path.rs:198-207) runs only under its check-nan / check-inf
    features; here it runs only when switched on, and names the tensor it found."""
    import torch
    q = torch.zeros(1, 2, 1, 4)
    v = torch.zeros(1, 2, 1, 6)
    v[0, 1, 0, 3] = float("nan")
    st = torch.zeros(1, 1, 4, 6)
    st[0, 0, 1, 1] = float("inf")
    inp = dn.DeltaInput(q, q, v, torch.zeros(1, 2, 1, 1), torch.zeros(1, 2, 1, 1), None, st)
    inp.sanity()  # off by default: shapes only
    try:
        dn.set_sanity_checks(nan=True, inf=False)
        with pytest.raises(dn.DeltaNonFiniteError, match="v holds NaN"):
            inp.sanity()
        v[0, 1, 0, 3] = 0.0
        inp.sanity()  # the Inf in the state passes while only check-nan is on
        dn.set_sanity_checks(nan=False, inf=True)
        with pytest.raises(dn.DeltaNonFiniteError, match="state holds Inf"):
            inp.sanity()
    finally:
        dn.set_sanity_checks(nan=False, inf=False)
    inp.sanity()


def test_host_entry_point_scratch_is_host_logic():
    a = _args(batch=10)
    need = abi.lib().dc_chunk_fwd_host_scratch_size(a)
    # two slots of 2 sequences each (10 sequences in up to 8 slices), every region 256-byte aligned
    seq = [9 * 2 * 4 * 4, 9 * 2 * 4 * 4, 9 * 2 * 6 * 4, 9 * 2 * 1 * 4, 9 * 2 * 1 * 4, 9 * 2 * 1 * 4,
           2 * 4 * 6 * 4, 9 * 2 * 6 * 4, 2 * 4 * 6 * 4]
    slot = sum(-(-2 * n // 256) * 256 for n in seq)
    # plus one slice's workspace for the fp32-accurate chunked path: 2 x 2 (batch, head) pairs of one
    # 32-row chunk, dk and dv padded to 8: W, K^, Q' and U [32][8], att [32][32], gam_L (4 floats)
    nch = 2 * 2 * 1
    ws = 4 * (3 * nch * 32 * 8 + nch * 32 * 8 + nch * 32 * 32 + 4)
    assert abi.lib().dc_chunk_workspace_size(_args(batch=2)) == ws
    assert need == 2 * slot + -(-ws // 256) * 256
    assert abi.lib().dc_chunk_fwd_host(a, 0x100000, need - 1, None) == abi.DC_EWORKSPACE
    assert abi.lib().dc_chunk_fwd_host(a, 0x100010, need, None) == abi.DC_EINVAL_ARG  # scratch not 256-aligned
    assert abi.lib().dc_chunk_fwd_host(_args(flags=abi.DC_FLAG_TEST_STALL), 0x100000, need, None) == abi.DC_EINVAL_ARG
    assert abi.lib().dc_chunk_fwd_host_scratch_size(_args(seq=0)) == 0


def test_backward_validation_and_workspace_are_host_logic():
    bw = abi.ChunkBwdArgs()
    bw.fwd = _args(dk=8, dv=8, seq=40)
    fake = 0x200000
    bw.d_y, bw.d_q, bw.d_k, bw.d_v = fake, fake + 4096, fake + 8192, fake + 12288
    bw.d_erase, bw.d_write, bw.d_g, bw.d_state = fake + 16384, fake + 20480, fake + 24576, fake + 28672
    # a log-decay per head takes the chunked backward: per 32-micro-step chunk (2 per (batch, head), 8 in
    # all; dk = dv = 8) W, K^, Q', U, V', dV' [32][8], att, T, A [32][32], gam_L, S and dS_next [8][8]
    nch = 2 * 2 * 2
    assert abi.lib().dc_chunk_bwd_workspace_size(bw) == 4 * (6 * nch * 32 * 8 + 3 * nch * 32 * 32 + nch + 2 * nch * 64)
    # the token-by-token one (DC_FLAG_RECURRENT, or per-channel log-decays): per (batch, head, 32-column
    # slice) the slice of the state at every 16th micro-step (ceil(40 / 16) = 3) and a 16-step buffer;
    # one slice (dv = 8): no partial sums
    rec = abi.ChunkBwdArgs.from_buffer_copy(bw)
    rec.fwd.flags = abi.DC_FLAG_RECURRENT
    assert abi.lib().dc_chunk_bwd_workspace_size(rec) == 2 * 2 * (3 + 16) * 8 * 32 * 4
    rec.fwd.flags, rec.fwd.g_w = 0, 8
    assert abi.lib().dc_chunk_bwd_workspace_size(rec) == 2 * 2 * (3 + 16) * 8 * 32 * 4
    assert abi.lib().dc_chunk_bwd(bw, None) == abi.DC_EWORKSPACE  # no workspace given
    bw.d_g = None
    assert abi.lib().dc_chunk_bwd(bw, None) == abi.DC_EINVAL_ARG  # gated forward needs d_g
    big = abi.ChunkBwdArgs()
    big.fwd = _args(dk=256, dv=8, erase_w=1)
    big.d_y = big.d_q = big.d_k = big.d_v = big.d_erase = big.d_write = big.d_g = big.d_state = fake
    assert abi.lib().dc_chunk_bwd(big, None) == abi.DC_EUNSUPPORTED


def test_out_norm_validation_is_host_logic():
    """dc_out_norm rejects bad arguments before any device work (OutNorm's shape asserts become codes)."""
    a = abi.OutNormArgs()
    a.rows, a.dv, a.in_dtype, a.out_dtype, a.eps = 4, 128, abi.DC_BF16, abi.DC_BF16, 1e-5
    a.y, a.gate, a.weight, a.out = 0x10000, 0x20000, 0x30000, 0x40000
    lib = abi.lib()
    bad = [("dv", 0, abi.DC_EINVAL_SHAPE), ("rows", -1, abi.DC_EINVAL_SHAPE), ("dv", 257, abi.DC_EUNSUPPORTED),
           ("eps", float("nan"), abi.DC_EINVAL_ARG), ("eps", -1.0, abi.DC_EINVAL_ARG),
           ("in_dtype", 5, abi.DC_EUNSUPPORTED_DTYPE), ("out_dtype", 5, abi.DC_EUNSUPPORTED_DTYPE),
           ("y", None, abi.DC_EINVAL_ARG), ("weight", None, abi.DC_EINVAL_ARG), ("out", None, abi.DC_EINVAL_ARG)]
    for name, value, code in bad:
        b = abi.OutNormArgs.from_buffer_copy(a)
        setattr(b, name, value)
        assert lib.dc_out_norm(b, None) == code, name
    empty = abi.OutNormArgs.from_buffer_copy(a)
    empty.rows, empty.y, empty.weight, empty.out = 0, None, None, None
    assert lib.dc_out_norm(empty, None) == abi.DC_OK  # nothing to do: no device touched
    assert lib.dc_out_norm(None, None) == abi.DC_EINVAL_ARG


def _norm_for(a, **over):
    n = abi.OutNormArgs()
    n.rows, n.dv, n.in_dtype, n.out_dtype, n.eps = a.batch * a.seq * a.heads, a.dv, a.out_dtype, a.out_dtype, 1e-5
    n.weight = 0x30000
    for k, v in over.items():
        setattr(n, k, v)
    return n


def test_chunk_out_norm_validation_and_fusion_are_host_logic():
    """dc_chunk_fwd_out_norm checks the norm against the prefill before any device work; its query says
    where the plain norm runs inside the tensor-core kernel's read-out."""
    lib = abi.lib()
    tc = _args(dk=128, dv=128, in_dtype=abi.DC_BF16, out_dtype=abi.DC_BF16)
    assert lib.dc_chunk_kernel_choice(tc) == 1
    assert lib.dc_chunk_fwd_out_norm_fused(tc, _norm_for(tc)) == 1
    assert lib.dc_chunk_fwd_out_norm_fused(tc, _norm_for(tc, gate=0x50000)) == 0           # gated norm: two kernels
    assert lib.dc_chunk_fwd_out_norm_fused(_args(), _norm_for(_args())) == 0               # CUDA-core prefill
    rec = _args(dk=128, dv=128, in_dtype=abi.DC_BF16, flags=abi.DC_FLAG_RECURRENT)
    assert lib.dc_chunk_fwd_out_norm_fused(rec, _norm_for(rec)) == 0
    bad = [(dict(y=0x60000), abi.DC_EINVAL_ARG), (dict(out=0x60000), abi.DC_EINVAL_ARG),
           (dict(eps=float("inf")), abi.DC_EINVAL_ARG), (dict(eps=-1.0), abi.DC_EINVAL_ARG),
           (dict(dv=64), abi.DC_EINVAL_SHAPE), (dict(rows=3), abi.DC_EINVAL_SHAPE),
           (dict(out_dtype=abi.DC_F32), abi.DC_EUNSUPPORTED_DTYPE),
           (dict(gate=0x50000, in_dtype=abi.DC_F32), abi.DC_EUNSUPPORTED_DTYPE),
           (dict(weight=None), abi.DC_EINVAL_ARG)]
    for over, code in bad:
        n = _norm_for(tc, **over)
        assert lib.dc_chunk_fwd_out_norm(tc, n, None) == code, over
        assert lib.dc_chunk_fwd_out_norm_fused(tc, n) == -code, over
    assert lib.dc_chunk_fwd_out_norm(tc, None, None) == abi.DC_EINVAL_ARG
    assert lib.dc_chunk_fwd_out_norm(_args(seq=0), _norm_for(tc), None) == abi.DC_EINVAL_SHAPE
    empty = _args(batch=0)
    assert lib.dc_chunk_fwd_out_norm(empty, _norm_for(empty, weight=None), None) == abi.DC_OK  # no device touched


def test_prologue_validation_is_host_logic():
    """dc_qkv_prologue rejects bad arguments before any device work (conv.rs / qkv.rs asserts as codes)."""
    a = abi.PrologueArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv, a.n_householder, a.conv_kernel = 2, 9, 2, 8, 8, 1, 4
    a.in_dtype = a.out_dtype = abi.DC_F32
    a.flags = abi.DC_PROLOGUE_CONV_SILU | abi.DC_PROLOGUE_L2
    a.x_stride = 2 * 8 * 2 + 2 * 8
    a.x, a.conv_weight, a.q, a.k, a.v = 0x10000, 0x20000, 0x30000, 0x40000, 0x50000
    a.window_in, a.window_out = 0x60000, 0x70000
    lib = abi.lib()
    bad = [("seq", 0, abi.DC_EINVAL_SHAPE), ("dk", 0, abi.DC_EINVAL_SHAPE), ("n_householder", 0, abi.DC_EINVAL_SHAPE),
           ("conv_kernel", 0, abi.DC_EINVAL_ARG), ("conv_kernel", 9, abi.DC_EUNSUPPORTED), ("dv", 129, abi.DC_EUNSUPPORTED),
           ("x_stride", 47, abi.DC_EINVAL_SHAPE), ("in_dtype", 7, abi.DC_EUNSUPPORTED_DTYPE), ("flags", 0x8, abi.DC_EINVAL_ARG),
           ("x", None, abi.DC_EINVAL_ARG), ("conv_weight", None, abi.DC_EINVAL_ARG), ("v", None, abi.DC_EINVAL_ARG),
           ("window_out", 0x60010, abi.DC_EINVAL_ARG)]  # the next window may not overlap the one being read
    for name, value, code in bad:
        b = abi.PrologueArgs.from_buffer_copy(a)
        setattr(b, name, value)
        assert lib.dc_qkv_prologue(b, None) == code, name
    assert lib.dc_qkv_prologue(None, None) == abi.DC_EINVAL_ARG


def test_gates_validation_is_host_logic():
    a = abi.GateArgs()
    a.rows, a.cols, a.x_stride, a.kind, a.in_dtype, a.group = 8, 16, 40, abi.DC_GATE_CHANNEL_DECAY, abi.DC_F32, 4
    a.scale, a.lo, a.hi = -5.0, 0.0, 1.0
    a.x, a.bias, a.a_log, a.out = 0x10000, 0x20000, 0x30000, 0x40000
    lib = abi.lib()
    bad = [("cols", 0, abi.DC_EINVAL_SHAPE), ("x_stride", 15, abi.DC_EINVAL_SHAPE), ("kind", 3, abi.DC_EINVAL_ARG),
           ("in_dtype", 4, abi.DC_EUNSUPPORTED_DTYPE), ("group", 3, abi.DC_EINVAL_SHAPE), ("scale", float("inf"), abi.DC_EINVAL_ARG),
           ("x", None, abi.DC_EINVAL_ARG), ("bias", None, abi.DC_EINVAL_ARG), ("a_log", None, abi.DC_EINVAL_ARG)]
    for name, value, code in bad:
        b = abi.GateArgs.from_buffer_copy(a)
        setattr(b, name, value)
        assert lib.dc_gates(b, None) == code, name
    b = abi.GateArgs.from_buffer_copy(a)
    b.kind, b.lo, b.hi = abi.DC_GATE_HEAD_DECAY, 2.0, 1.0
    assert lib.dc_gates(b, None) == abi.DC_EINVAL_ARG  # clamp range upside down
    b = abi.GateArgs.from_buffer_copy(a)
    b.rows, b.x, b.out = 0, None, None
    assert lib.dc_gates(b, None) == abi.DC_OK
