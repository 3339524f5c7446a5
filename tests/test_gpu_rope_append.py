"""GPU parity of the fused rotary embedding + KV append: q_out and the pool
rows bit-identical to the oracle (pinned to transformers on CPU) and to
transformers' apply_rotary_pos_emb run on the GPU, plus the plain append of v."""
import pytest
import torch

import pagedkv
from oracle import paged_ref
from pagedkv import _native

pytestmark = pytest.mark.gpu


def _cos_sin(n, d, dtype, g):
    pos = torch.randint(0, 32768, (n,), generator=g).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat((pos[:, None] * inv[None, :],) * 2, dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _case(dev, dtype, hq, hkv, d, nb=32, bs=16, n=21, fused=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    if fused:  # q, k, v as views of one fused qkv projection (strided rows)
        qkv = (torch.randn(n, (hq + 2 * hkv) * d, generator=g) * 2).to(dtype)
        q = qkv[:, : hq * d].view(n, hq, d)
        k = qkv[:, hq * d : (hq + hkv) * d].view(n, hkv, d)
        v = qkv[:, (hq + hkv) * d :].view(n, hkv, d)
    else:
        q = (torch.randn(n, hq, d, generator=g) * 2).to(dtype)
        k = (torch.randn(n, hkv, d, generator=g) * 2).to(dtype)
        v = torch.randn(n, hkv, d, generator=g).to(dtype)
    cos, sin = _cos_sin(n, d, dtype, g)
    kc = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    vc = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int64)
    slots[3] = -1  # padding token: no write
    return q, k, v, cos, sin, kc, vc, slots


def _expected(q, k, v, cos, sin, kc, vc, slots):
    qe = paged_ref.rope_ref(q, cos, sin)
    ke = paged_ref.rope_ref(k, cos, sin)
    kc, vc = kc.clone(), vc.clone()
    bs = kc.shape[1]
    for i, s in enumerate(slots.tolist()):
        if s >= 0:
            kc[s // bs, s % bs] = ke[i]
            vc[s // bs, s % bs] = v[i]
    return qe, kc, vc


def _bits(t):
    return t.detach().cpu().view(torch.int16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (56, 8, 128), (8, 1, 32), (4, 2, 256)])
@pytest.mark.parametrize("fused", [False, True])
def test_append_rope_vs_oracle(cuda_ready, dtype, hq, hkv, d, fused):
    q, k, v, cos, sin, kc, vc, slots = _case(cuda_ready, dtype, hq, hkv, d, fused=fused, seed=hq + d)
    qe, kce, vce = _expected(q, k, v, cos, sin, kc, vc, slots)
    dk, dv = kc.to(cuda_ready), vc.to(cuda_ready)
    qo = pagedkv.kv_append_rope(q.to(cuda_ready), k.to(cuda_ready), v.to(cuda_ready), cos.to(cuda_ready),
                                sin.to(cuda_ready), dk, dv, slots.to(cuda_ready))
    assert torch.equal(_bits(qo), _bits(qe))
    assert torch.equal(_bits(dk), _bits(kce)) and torch.equal(_bits(dv), _bits(vce))


def test_append_rope_matches_transformers_on_gpu(cuda_ready):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    q, k, v, cos, sin, kc, vc, slots = _case(cuda_ready, torch.float16, 14, 2, 64, seed=5)
    q, k, v, cos, sin = (t.to(cuda_ready) for t in (q, k, v, cos, sin))
    rq, rk = apply_rotary_pos_emb(q[:, :, None, :], k[:, :, None, :], cos[:, None, :], sin[:, None, :])
    dk, dv = kc.to(cuda_ready), vc.to(cuda_ready)
    qo = pagedkv.kv_append_rope(q, k, v, cos, sin, dk, dv, slots.to(cuda_ready))
    assert torch.equal(_bits(qo), _bits(rq[:, :, 0, :]))
    bs = kc.shape[1]
    for i, s in enumerate(slots.tolist()):
        if s >= 0:
            assert torch.equal(_bits(dk[s // bs, s % bs]), _bits(rk[i, :, 0, :]))


def test_append_rope_in_place_unaligned_and_bad_slot(cuda_ready):
    q, k, v, cos, sin, kc, vc, slots = _case(cuda_ready, torch.float16, 14, 2, 64, seed=9)
    qe, kce, vce = _expected(q, k, v, cos, sin, kc, vc, slots)
    # in place (q_out is q), sources starting one element in (element-wise path)
    qbuf = torch.zeros(q.numel() + 1, dtype=q.dtype)
    qbuf[1:] = q.reshape(-1)
    dq = qbuf.to(cuda_ready)[1:].view(q.shape)
    dk, dv = kc.to(cuda_ready), vc.to(cuda_ready)
    out = pagedkv.kv_append_rope(dq, k.to(cuda_ready), v.to(cuda_ready), cos.to(cuda_ready), sin.to(cuda_ready),
                                 dk, dv, slots.to(cuda_ready), q_out=dq)
    assert out.data_ptr() == dq.data_ptr()
    assert torch.equal(_bits(dq), _bits(qe))
    assert torch.equal(_bits(dk), _bits(kce)) and torch.equal(_bits(dv), _bits(vce))
    pagedkv.read_error_flags(cuda_ready, clear=True)
    bad = slots.clone()
    bad[0] = kc.shape[0] * kc.shape[1] + 5
    pagedkv.kv_append_rope(q.to(cuda_ready), k.to(cuda_ready), v.to(cuda_ready), cos.to(cuda_ready),
                           sin.to(cuda_ready), dk, dv, bad.to(cuda_ready))
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_SLOT_RANGE


@pytest.mark.parametrize("hq,hkv,d,n,fused,dtype", [
    (14, 2, 64, 42_100, False, torch.float16),   # 5 rows per thread: groups of 5, 5, 5, 3
    (14, 2, 64, 160_000, True, torch.bfloat16),  # a whole token per thread (18 rows)
    (4, 2, 256, 40_000, False, torch.float16),   # a whole token per thread (8 rows)
    (56, 8, 128, 5_300, True, torch.float16),    # 5 rows per thread, 72 rows: last group of 2
])
def test_append_rope_bulk_row_groups_vs_oracle(cuda_ready, hq, hkv, d, n, fused, dtype):
    """Launches large enough that each thread takes several head rows of one
    token (the rows-per-thread split of the bulk path), with padding and
    ragged last groups: still bit-identical to the oracle."""
    bs = 16
    nb = (n + bs - 1) // bs + 4
    q, k, v, cos, sin, kc, vc, slots = _case(cuda_ready, dtype, hq, hkv, d, nb=nb, bs=bs, n=n, fused=fused,
                                             seed=n % 97)
    slots[::1000] = -1  # padding tokens spread over the launch
    qe = paged_ref.rope_ref(q, cos, sin)
    ke = paged_ref.rope_ref(k, cos, sin)
    live = slots >= 0
    kce, vce = kc.clone(), vc.clone()
    kce.view(-1, hkv, d)[slots[live]] = ke[live]
    vce.view(-1, hkv, d)[slots[live]] = v[live]
    dk, dv = kc.to(cuda_ready), vc.to(cuda_ready)
    qo = pagedkv.kv_append_rope(q.to(cuda_ready), k.to(cuda_ready), v.to(cuda_ready), cos.to(cuda_ready),
                                sin.to(cuda_ready), dk, dv, slots.to(cuda_ready))
    assert torch.equal(_bits(qo), _bits(qe))
    assert torch.equal(_bits(dk), _bits(kce)) and torch.equal(_bits(dv), _bits(vce))
    assert pagedkv.read_error_flags(cuda_ready) == 0
