"""CPU restatement of the reference's one-token MLA attention -- TEST
INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's baseline / reference legs
use it as the checker; the product never imports it).

Restated from src/pcketlm/native/ds_forward.cpp of the reference:
  mla_attention_flash  <- ds_mla_attention_flash_forward  :517-597
  attention_block      <- ds_attention_block_forward_f32  :647-782
                          (rms_norm_inplace_f32 :612-620,
                           apply_rope_groups_inplace_f32 :622-645)
in fp32 with the reference's per-position online softmax (running max,
rescaled running sum and latent sums, exp(old - new) = 0 at the start),
vectorised over heads: every head's recurrence is the reference's, only the
summation order inside each dot product is torch's.  Pinned against the
reference compiled from those sources (oracle/_ref/ds_forward.so) by
tests/test_mla_host.py and by the golden vectors tests/golden/mla_*.pt.
"""

from __future__ import annotations

import torch


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().contiguous().to(torch.float32)


def rms_norm(values: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """ds_forward.cpp:612-620: values * (1 / sqrt(mean(values^2) + eps)) * weight."""
    sum_sq = (values * values).sum()
    inv = 1.0 / torch.sqrt(sum_sq / float(values.numel()) + torch.tensor(eps, dtype=torch.float32))
    return (values * inv) * weight


def rope_groups(values: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """ds_forward.cpp:622-645 on [groups, rope]: pairs (2p, 2p + 1) rotated by
    (cos[p], sin[p]); an odd rope width is left as it is."""
    rope = int(values.shape[-1])
    if rope <= 0 or rope % 2:
        return values.clone()
    x0, x1 = values[..., 0::2], values[..., 1::2]
    out = torch.empty_like(values)
    out[..., 0::2] = x0 * cos - x1 * sin
    out[..., 1::2] = x0 * sin + x1 * cos
    return out


def mla_attention_flash(q_nope: torch.Tensor, q_pe: torch.Tensor, kv_cache: torch.Tensor, pe_cache: torch.Tensor,
                        wkv_b: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """[heads, nope], [heads, rope], [L, R], [L, rope], [heads, nope + v, R] -> [heads, v]."""
    qn, qp, kv, pe, w = _f32(q_nope), _f32(q_pe), _f32(kv_cache), _f32(pe_cache), _f32(wkv_b)
    heads, nope = int(qn.shape[0]), int(qn.shape[1])
    rope = int(qp.shape[1])
    R = int(kv.shape[1])
    q_abs = torch.einsum("hd,hdc->hc", qn, w[:, :nope])  # :550-557
    latent = torch.zeros((heads, R), dtype=torch.float32)
    running_max = torch.full((heads,), float("-inf"), dtype=torch.float32)
    running_sum = torch.zeros((heads,), dtype=torch.float32)
    scale = torch.tensor(softmax_scale, dtype=torch.float32)
    for pos in range(int(kv.shape[0])):  # :562-580
        score = q_abs @ kv[pos]
        if rope > 0:
            score = score + qp @ pe[pos]
        score = score * scale
        new_max = torch.where(running_max > score, running_max, score)
        old_scale = torch.where(torch.isfinite(running_max), torch.exp(running_max - new_max),
                                torch.zeros_like(running_max))
        score_scale = torch.exp(score - new_max)
        latent = latent * old_scale[:, None] + kv[pos][None, :] * score_scale[:, None]
        running_sum = running_sum * old_scale + score_scale
        running_max = new_max
    inv = torch.where(running_sum > 0, 1.0 / running_sum, torch.zeros_like(running_sum))  # :581-585
    latent = latent * inv[:, None]
    return torch.einsum("hc,hdc->hd", latent, w[:, nope:]).contiguous()  # :587-595


def attention_block(hidden, q_a, q_b, kv_a, kv_b, o_w, q_norm, kv_norm, previous_kv, previous_pe, cos, sin, *,
                    q_lora_rank: int, kv_lora_rank: int, num_heads: int, qk_nope_dim: int, qk_rope_dim: int,
                    v_head_dim: int, rms_eps: float, softmax_scale: float):
    """ds_forward.cpp:691-782 -> (hidden_out [H], (next_kv [L, R], next_pe [L, rope]))."""
    x = _f32(hidden).reshape(-1)
    nope, rope, R, heads = qk_nope_dim, qk_rope_dim, kv_lora_rank, num_heads
    cos_f, sin_f = _f32(cos).reshape(-1), _f32(sin).reshape(-1)
    q_low = rms_norm(_f32(q_a) @ x, _f32(q_norm).reshape(-1), rms_eps)  # :709-710
    q = (_f32(q_b) @ q_low).reshape(heads, nope + rope)  # :712-724
    q_nope, q_pe = q[:, :nope], q[:, nope:]
    if rope > 0:
        q_pe = rope_groups(q_pe, cos_f, sin_f)  # :725-726
    kv_row = _f32(kv_a) @ x  # :743-755
    new_kv = rms_norm(kv_row[:R], _f32(kv_norm).reshape(-1), rms_eps)
    new_pe = rope_groups(kv_row[R:].reshape(1, rope), cos_f, sin_f).reshape(-1) if rope > 0 else kv_row[R:]
    prev_kv = torch.zeros((0, R)) if previous_kv is None else _f32(previous_kv).reshape(-1, R)
    prev_pe = torch.zeros((0, rope)) if previous_pe is None else _f32(previous_pe).reshape(-1, rope)
    next_kv = torch.cat([prev_kv, new_kv.reshape(1, R)], 0)  # :727-742
    next_pe = torch.cat([prev_pe, new_pe.reshape(1, rope)], 0)
    heads_out = mla_attention_flash(q_nope, q_pe, next_kv, next_pe,
                                    _f32(kv_b).reshape(heads, nope + v_head_dim, R), softmax_scale)  # :758-775
    return _f32(o_w) @ heads_out.reshape(-1), (next_kv, next_pe)  # :777
