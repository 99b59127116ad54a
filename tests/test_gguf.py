"""GGUF ingestion (moe_gguf_*): expert stacks read from an on-disk GGUF file through the library's native
reader must be the very bytes that were written, laid out as the stacked [E, N, K] tensors the
reference's provider receives (provider.rs:367) and slices per expert (expert.rs:123-145).

The files are written with the gguf Python package (the llama.cpp project's published GGUF writer),
which the library shares no code with. The CPU tests read headers, metadata and tensors; the GPU test
builds a layer from the file and from the same bytes in memory and requires bit-identical outputs.
"""

import numpy as np
import pytest

from oracle import oracle as O

gguf = pytest.importorskip("gguf")

E, K_TOP, H, I = 8, 2, 256, 256


def _stacks(rng, dtype):
    out = []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        q, _ = O.quantize(dtype, rng.normal(0, 0.02, shape).astype(np.float32))
        out.append(q)
    return out


def write_model(path, seed=1, router_dtype=np.float32, types=(O.DT_Q8_0, O.DT_Q4_K)):
    """A two-layer MoE GGUF (one expert type per layer) plus its source bytes."""
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(str(path), "qwen3moe")
    w.add_uint32("qwen3moe.expert_count", E)
    w.add_uint32("qwen3moe.expert_used_count", K_TOP)
    w.add_uint32("qwen3moe.block_count", len(types))
    gtype = {O.DT_Q8_0: gguf.GGMLQuantizationType.Q8_0, O.DT_Q4_K: gguf.GGMLQuantizationType.Q4_K,
             O.DT_BF16: gguf.GGMLQuantizationType.BF16}
    src = []
    for li, dt in enumerate(types):
        q = _stacks(rng, dt)
        router = rng.normal(0, 0.02, (E, H)).astype(np.float32)
        for name, b, shape in (("ffn_gate_exps", q[0], (E, I, H)), ("ffn_up_exps", q[1], (E, I, H)),
                               ("ffn_down_exps", q[2], (E, H, I))):
            per = {O.DT_Q8_0: (32, 34), O.DT_Q4_K: (256, 144), O.DT_BF16: (1, 2)}[dt]
            raw = b.reshape(shape[0], shape[1], shape[2] // per[0] * per[1])
            w.add_tensor(f"blk.{li}.{name}.weight", raw, raw_dtype=gtype[dt])  # byte shape [E, N, row bytes]
        if router_dtype == np.float32:
            w.add_tensor(f"blk.{li}.ffn_gate_inp.weight", router)
        else:
            w.add_tensor(f"blk.{li}.ffn_gate_inp.weight", O.f32_to_bf16(router).reshape(E, H).view(np.uint8),
                         raw_dtype=gguf.GGMLQuantizationType.BF16)
        src.append((dt, q, router))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return src


@pytest.fixture()
def model(tmp_path):
    path = tmp_path / "moe.gguf"
    return path, write_model(path)


def test_reads_metadata_and_tensor_table(model):
    import moe_b200 as M

    path, src = model
    with M.GGUFFile(str(path)) as f:
        assert f.get_str("general.architecture") == "qwen3moe"
        assert f.get_int("qwen3moe.expert_count") == E and f.get_int("qwen3moe.expert_used_count") == K_TOP
        assert f.get_int("no.such.key") is None
        names = set(f.tensor_names())
        for li in range(2):
            for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps", "ffn_gate_inp"):
                assert f"blk.{li}.{n}.weight" in names
        t, dims, view = f.tensor("blk.0.ffn_gate_exps.weight")
        assert t == 8 and dims == (H, I, E)  # Q8_0; dims[0] fastest
        assert np.array_equal(view, src[0][1][0])
        t, dims, view = f.tensor("blk.1.ffn_down_exps.weight")
        assert t == 12 and dims == (I, H, E)  # Q4_K
        assert np.array_equal(view, src[1][1][2])


@pytest.mark.parametrize("router_dtype", [np.float32, np.uint16])
def test_layer_context_points_at_the_file_bytes(tmp_path, router_dtype):
    import moe_b200 as M

    path = tmp_path / "m.gguf"
    src = write_model(path, seed=3, router_dtype=router_dtype)
    with M.GGUFFile(str(path)) as f:
        for li, (dt, q, router) in enumerate(src):
            ctx = f.layer_context(li, device=0, max_tokens=16)
            assert ctx.wdtype == dt and ctx.config.num_experts == E and ctx.config.num_experts_per_tok == K_TOP
            assert ctx.config.hidden_size == H and ctx.config.moe_intermediate_size == I
            for got, want in zip((ctx.gate, ctx.up, ctx.down), q):
                assert np.array_equal(got, want)
            # expert e's bytes are the e-th contiguous range of each stack (expert.rs:123-145)
            b0, b1 = O.expert_range(dt, E, I, H, 5)
            assert np.array_equal(ctx.gate[b0:b1], q[0][b0:b1])
            assert np.array_equal(ctx.router_weight, O.f32_to_bf16(router).reshape(E, H))


def test_rejects_malformed_files(tmp_path, model):
    import moe_b200 as M

    path, _ = model
    data = open(path, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + data[4:])
    with pytest.raises(M.MoeError, match="magic"):
        M.GGUFFile(str(bad))
    bad.write_bytes(data[: len(data) // 2])  # tensor data cut off
    with pytest.raises(M.MoeError, match="past the end|truncated"):
        M.GGUFFile(str(bad))
    bad.write_bytes(data[:40])  # metadata cut off
    with pytest.raises(M.MoeError):
        M.GGUFFile(str(bad))
    with pytest.raises(M.MoeError, match="cannot open"):
        M.GGUFFile(str(tmp_path / "missing.gguf"))
    with M.GGUFFile(str(path)) as f:
        with pytest.raises(M.MoeError, match="no tensor"):
            f.layer_context(7, device=0)


def test_rejects_mixed_expert_types(tmp_path):
    """One layer runs one weight type (the reference's GGUF has layers whose down differs from gate/up,
    tests.rs:85, which its candle path runs per projection; this library does not)."""
    import moe_b200 as M

    rng = np.random.default_rng(0)
    path = tmp_path / "mixed.gguf"
    w = gguf.GGUFWriter(str(path), "qwen3moe")
    q8 = _stacks(rng, O.DT_Q8_0)
    q4 = _stacks(rng, O.DT_Q4_K)
    w.add_tensor("blk.0.ffn_gate_exps.weight", q8[0].reshape(E, I, -1), raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    w.add_tensor("blk.0.ffn_up_exps.weight", q8[1].reshape(E, I, -1), raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    w.add_tensor("blk.0.ffn_down_exps.weight", q4[2].reshape(E, H, -1), raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with M.GGUFFile(str(path)) as f:
        with pytest.raises(M.MoeError, match="mixes weight types"):
            f.layer_context(0, device=0, top_k=2)


@pytest.mark.gpu
def test_layer_from_gguf_matches_layer_from_memory(model):
    """The same stacks through moe_layer_create from the file mapping and from numpy memory: outputs
    bit-identical (and the router too)."""
    import torch

    import moe_b200 as M

    path, src = model
    rng = np.random.default_rng(9)
    T = 24
    x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
        .view(torch.bfloat16).cuda()
    with M.GGUFFile(str(path)) as f:
        for li, (dt, q, router) in enumerate(src):
            a = M.RoutedExpertsProvider().build(f.layer_context(li, device=0, max_tokens=T))
            cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I)
            b = M.RoutedExpertsProvider().build(M.ExpertLoadContext(
                layer=li, device=0, config=cfg, wdtype=dt, gate=q[0], up=q[1], down=q[2],
                router_weight=O.f32_to_bf16(router).reshape(E, H), max_tokens=T))
            ia, wa = a.route(x)
            ib, wb = b.route(x)
            assert torch.equal(ia, ib) and torch.equal(wa, wb)
            assert torch.equal(a.forward(x, wa, ia), b.forward(x, wb, ib))
            a.check()
            b.check()
            a.close()
            b.close()
