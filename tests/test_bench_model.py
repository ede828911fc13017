"""The work models behind bench.py's roofline numbers, checked on CPU against
the tensor list of the synthetic model (the architecture the engine loads):
the algorithmic weight bytes one decode token streams, and the FLOPs of a
prefill. These are the numerators of `roofline.achieved` and
`prefill.tflops`."""

import math

import bench
import synth_gguf as sg


def _q6_tensors():
    return [(name, ne) for name, typ, ne, _ in sg.tensor_plan() if typ == sg.GGML_Q6_K]


def _q6_bytes(ne):
    rows = math.prod(ne[1:])
    return rows * (ne[0] // sg.QK_K) * sg.Q6_BYTES


def test_decode_weight_bytes_match_the_tensor_list():
    # every dense matrix once, the routed experts' share (top 4 of 32), and the
    # tied embedding once as the lm_head
    total = 0
    for name, ne in _q6_tensors():
        b = _q6_bytes(ne)
        total += b * sg.N_USED // sg.N_EXPERT if "_exps" in name else b
    assert bench.decode_bytes_per_token(512)["q6"] == total


def test_decode_bytes_count_kv_reads_per_position():
    a, b = bench.decode_bytes_per_token(512), bench.decode_bytes_per_token(513)
    n_attn = len(sg.ATTN_LAYERS)
    # fp16 K and V of every KV head of every attention layer, one more position
    assert b["kv"] - a["kv"] == n_attn * 2 * sg.KV_HEADS * sg.HEAD_DIM * 2


def test_router_bytes():
    n_moe = sg.N_LAYERS - sg.DENSE_LEAD
    assert bench.decode_bytes_per_token(1)["router"] == n_moe * sg.DIM * sg.N_EXPERT * 4


def test_prefill_flops_match_the_tensor_list():
    n = 3840
    mac_tok = 0
    for name, ne in _q6_tensors():
        if name == "token_embd.weight":
            continue  # the lm_head runs for the last token only
        macs = ne[0] * math.prod(ne[1:])
        mac_tok += macs * sg.N_USED // sg.N_EXPERT if "_exps" in name else macs
    # causal attention: token i attends to i+1 positions, QK^T and PV, every head
    attn_macs = len(sg.ATTN_LAYERS) * sg.HEADS * sg.HEAD_DIM * 2 * (n * (n + 1) // 2)
    lm_head = sg.DIM * sg.VOCAB
    expected = 2.0 * (mac_tok * n + attn_macs + lm_head)
    assert math.isclose(bench.prefill_flops(n), expected, rel_tol=1e-12)


def test_bench_constants_follow_the_model():
    assert (bench.DIM, bench.VOCAB) == (sg.DIM, sg.VOCAB)
    assert bench.N_ATTN == len(sg.ATTN_LAYERS)
    assert bench.N_CONV == sg.N_LAYERS - len(sg.ATTN_LAYERS)
    assert bench.N_DENSE == sg.DENSE_LEAD
    assert bench.N_MOE == sg.N_LAYERS - sg.DENSE_LEAD
