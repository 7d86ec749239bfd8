"""CPU oracle for the ring context-parallel attention hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA product
path is compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The
product package (``hcp_vllm_plugin_b200``) never imports it and has no CPU
fallback.

It restates, in numpy float32, the reference plugin's fp32 torch path — the
path selected by ``HCP_RING_IMPL=torch`` / ``HCP_RING_MERGE=torch`` — and the
per-request ring driver of ``HcpRingAttentionImpl.forward``.  File:line
citations are relative to the reference project (stark-sim/hcp-vllm-plugin).

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
``_attn_with_lse`` / ``_lse_merge`` / ``HcpRingAttentionImpl.forward`` on CPU
and committed their inputs and outputs; ``tests/test_oracle_golden.py`` checks
this module against those fixtures.

Layouts (same as the reference unless stated):
  q            [Tq, H, D]
  k, v         [Tk, Hkv, D]
  out          [Tq, H, D] float32
  lse          [H, Tq]   float32, natural log
  paged cache  [num_blocks, Hkv, block_size, 2*D]; K = [..., :D], V = [..., D:]
               (the layout ``hcp_vllm_plugin/file_connector.py:14-16, 175-179``
               documents; the reference backend itself declares
               ``[num_blocks, 2, block_size, Hkv, D]``, ``ring_backend.py:458``)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

LN2 = math.log(2.0)


# ---------------------------------------------------------------------------
# 16-bit float helpers (numpy has no bfloat16)
# ---------------------------------------------------------------------------
def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen raw bfloat16 bit patterns (uint16) to float32 exactly."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (round-to-nearest-even), return uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---------------------------------------------------------------------------
# Attention with LSE and the LSE merge
# ---------------------------------------------------------------------------
def attn_with_lse(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    scale: float,
    q_pos0_in_kv: int | None,
    window: int | None = None,
    q_block: int = 256,
) -> tuple[np.ndarray, np.ndarray]:
    """Attention with explicit natural-log logsumexp, fp32.

    Restates ``_attn_with_lse`` (``hcp_vllm_plugin/ring_backend.py:366-406``):
    GQA by repeating each KV head over its ``H // Hkv`` query heads
    (``:384-388``), scores ``q.k * scale`` in fp32 (``:389-390``), causal mask
    ``j <= q_pos0_in_kv + i`` with optional sliding window ``j > qpos - w``
    (``:391-398``), max-shifted exp, normalised output and
    ``lse = max + log(sum)`` (``:399-405``).

    ``q_pos0_in_kv`` is the position of query row 0 in this KV block's frame,
    ``None`` for non-causal.  Query rows are independent, so they are processed
    ``q_block`` at a time to bound memory (the reference materialises the whole
    ``[H, Tq, Tk]`` score tensor, which is too large at long lengths).

    Returns (out [Tq, H, D] float32, lse [H, Tq] float32).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    tq, num_heads, head_dim = q.shape
    tk, num_kv_heads, _ = k.shape
    group = num_heads // num_kv_heads
    out = np.empty((tq, num_heads, head_dim), dtype=np.float32)
    lse = np.empty((num_heads, tq), dtype=np.float32)
    # [Hkv, Tk, D] views for batched matmul per KV head.
    kh = np.ascontiguousarray(k.transpose(1, 0, 2))
    vh = np.ascontiguousarray(v.transpose(1, 0, 2))
    j = np.arange(tk)[None, :]
    for r0 in range(0, tq, q_block):
        r1 = min(tq, r0 + q_block)
        # [H, rows, D] -> [Hkv, group*rows, D]
        qb = q[r0:r1].transpose(1, 0, 2).reshape(num_kv_heads, group * (r1 - r0), head_dim)
        s = np.matmul(qb, kh.transpose(0, 2, 1)) * np.float32(scale)  # [Hkv, g*rows, Tk]
        s = s.reshape(num_heads, r1 - r0, tk)
        if q_pos0_in_kv is not None:
            qpos = q_pos0_in_kv + np.arange(r0, r1)[:, None]
            mask = j <= qpos
            if window is not None:
                mask &= j > qpos - window
            s = np.where(mask[None], s, np.float32(-np.inf))
        m = s.max(axis=-1)  # [H, rows]
        p = np.exp(s - m[..., None])
        denom = p.sum(axis=-1)  # [H, rows]
        o = np.matmul(
            p.reshape(num_kv_heads, group * (r1 - r0), tk), vh
        ).reshape(num_heads, r1 - r0, head_dim)
        o = o / denom[..., None]
        out[r0:r1] = o.transpose(1, 0, 2)
        lse[:, r0:r1] = m + np.log(denom)
    return out, lse


def lse_merge(o1, lse1, o2, lse2) -> np.ndarray:
    """Online-softmax merge of two partial attentions over disjoint KV sets.

    Restates ``_lse_merge`` (``hcp_vllm_plugin/ring_backend.py:409-421``):
    ``w_i = exp(lse_i - max)``, ``out = (o1 w1 + o2 w2) / (w1 + w2)``.
    o: [Tq, H, D], lse: [H, Tq].
    """
    o1 = np.asarray(o1, dtype=np.float32)
    o2 = np.asarray(o2, dtype=np.float32)
    lse1 = np.asarray(lse1, dtype=np.float32)
    lse2 = np.asarray(lse2, dtype=np.float32)
    m = np.maximum(lse1, lse2)
    w1 = np.exp(lse1 - m).T[..., None]
    w2 = np.exp(lse2 - m).T[..., None]
    return (o1 * w1 + o2 * w2) / (w1 + w2)


def merge_pair(o1, lse1, o2, lse2) -> tuple[np.ndarray, np.ndarray]:
    """Merge two partials and also return the merged LSE.

    Restates ``_merge_pair`` (``hcp_vllm_plugin/ring_decode.py:46-61``): the
    output is ``merge_attn_states`` (same formula as :func:`lse_merge`) and the
    merged LSE is ``m + log(exp(lse1 - m) + exp(lse2 - m))`` (``:59-60``).
    """
    out = lse_merge(o1, lse1, o2, lse2)
    lse1 = np.asarray(lse1, dtype=np.float32)
    lse2 = np.asarray(lse2, dtype=np.float32)
    m = np.maximum(lse1, lse2)
    lse = m + np.log(np.exp(lse1 - m) + np.exp(lse2 - m))
    return out, lse


def merge_attn_states(prefix_o, prefix_lse, suffix_o, suffix_lse):
    """vLLM ``merge_attn_states(out, prefix_output, prefix_lse, suffix_output,
    suffix_lse)`` restated (third-party, vLLM 0.22.0
    ``vllm/v1/attention/ops/triton_merge_attn_states.py``): a ``+inf`` LSE is
    treated as ``-inf`` (an empty partial), then the same max-shifted weighted
    average as :func:`lse_merge`.  Returns (out, merged lse).

    Called by the reference at ``ring_backend.py:349-356`` (prefix = peer,
    suffix = local) and ``ring_decode.py:55-58``.
    """
    p_lse = np.where(np.isposinf(prefix_lse), -np.inf, prefix_lse).astype(np.float32)
    s_lse = np.where(np.isposinf(suffix_lse), -np.inf, suffix_lse).astype(np.float32)
    m = np.maximum(p_lse, s_lse)
    m_safe = np.where(np.isneginf(m), 0.0, m).astype(np.float32)
    wp = np.exp(p_lse - m_safe)
    ws = np.exp(s_lse - m_safe)
    tot = wp + ws
    inv = np.where(tot > 0, 1.0 / np.where(tot > 0, tot, 1.0), 0.0).astype(np.float32)
    out = (np.asarray(prefix_o, np.float32) * (wp * inv).T[..., None]
           + np.asarray(suffix_o, np.float32) * (ws * inv).T[..., None])
    lse = np.where(tot > 0, np.log(np.where(tot > 0, tot, 1.0)) + m_safe, -np.inf)
    return out, lse.astype(np.float32)


# ---------------------------------------------------------------------------
# Paged KV cache
# ---------------------------------------------------------------------------
def paged_gather(cache: np.ndarray, block_row: np.ndarray, tk: int) -> tuple[np.ndarray, np.ndarray]:
    """Contiguous K, V [tk, Hkv, D] of one request out of the paged cache.

    The reference gathers ``key_cache[block_table[r, :nb]]`` and reshapes
    (``ring_backend.py:616-624``); here the cache is
    ``[num_blocks, Hkv, block_size, 2*D]`` with K in the first D lanes of the
    last dimension and V in the second (``file_connector.py:175-179``).
    """
    _, hkv, bs, d2 = cache.shape
    d = d2 // 2
    nb = (tk + bs - 1) // bs
    blocks = cache[np.asarray(block_row[:nb], dtype=np.int64)]  # [nb, Hkv, bs, 2D]
    kv = blocks.transpose(0, 2, 1, 3).reshape(nb * bs, hkv, d2)[:tk]
    return kv[..., :d], kv[..., d:]


def kv_cache_update(cache: np.ndarray, key: np.ndarray, value: np.ndarray,
                    slot_mapping: np.ndarray) -> None:
    """Scatter new K/V rows into the paged cache in place.

    Restates ``do_kv_cache_update`` (``ring_backend.py:501-539``: block index
    ``slot // block_size``, offset ``slot % block_size``, ``:532-537``) in the
    ``[num_blocks, Hkv, block_size, 2*D]`` layout (``file_connector.py:175-179``).
    Slots < 0 are padding and are skipped (vLLM marks padded tokens with -1).
    """
    _, _, bs, d2 = cache.shape
    d = d2 // 2
    slot_mapping = np.asarray(slot_mapping, dtype=np.int64)
    n = slot_mapping.shape[0]
    for i in range(n):
        s = int(slot_mapping[i])
        if s < 0:
            continue
        b, o = divmod(s, bs)
        cache[b, :, o, :d] = key[i]
        cache[b, :, o, d:] = value[i]


def kv_cache_gather(cache: np.ndarray, slot_mapping: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """K, V [n, Hkv, D] of the given slots out of the paged cache.

    Restates the producer's pool -> chunk extraction of
    ``HcpRingKvConnector.save_kv_layer`` (``ring_connector.py:906-910``:
    ``kv_layer[slot // block_size, :, slot % block_size]``) in the
    ``[num_blocks, Hkv, block_size, 2*D]`` layout; rows of slots outside the
    cache (or negative) are zeros.
    """
    nb, hkv, bs, d2 = cache.shape
    d = d2 // 2
    slot_mapping = np.asarray(slot_mapping, dtype=np.int64)
    k = np.zeros((slot_mapping.shape[0], hkv, d), cache.dtype)
    v = np.zeros_like(k)
    for i, s in enumerate(slot_mapping):
        if 0 <= s < nb * bs:
            b, o = divmod(int(s), bs)
            k[i] = cache[b, :, o, :d]
            v[i] = cache[b, :, o, d:]
    return k, v


# ---------------------------------------------------------------------------
# The per-request ring driver of HcpRingAttentionImpl.forward
# ---------------------------------------------------------------------------
@dataclass
class RingRequestPlan:
    """How the reference's ``forward`` splits one request (``ring_backend.py:611-832``)."""

    q_start: int          # first query row of the request in the batch
    tq: int               # query rows
    tk: int               # seq_len (keys in the paged cache incl. the peer prefix)
    qpos0: int            # global position of query 0 = tk - tq  (:627)
    peer_end: int         # keys of the peer prefix (0 = vanilla path)
    peer_source: str      # "staged" | "split" | "none"
    n_a: int              # queries still inside the peer region (:811)


def plan_request(q_start: int, tq: int, tk: int, staged_len: int | None, split: int) -> RingRequestPlan:
    """Restates the per-request bookkeeping of ``forward`` (``ring_backend.py:611-627,
    773-781, 811``): staged peer KV takes precedence over ``HCP_RING_SPLIT_TOKENS``."""
    qpos0 = tk - tq
    if staged_len is not None:
        peer_end, src = min(staged_len, tk), "staged"
    elif split > 0:
        peer_end, src = min(split, tk), "split"
    else:
        peer_end, src = 0, "none"
    n_a = max(0, min(tq, peer_end - qpos0)) if peer_end > 0 else 0
    return RingRequestPlan(q_start, tq, tk, qpos0, peer_end, src, n_a)


@dataclass
class RingBatch:
    """Inputs of one attention-layer call, as vLLM hands them to ``forward``."""

    query: np.ndarray                 # [num_tokens, H, D] float32 (bf16-valued)
    cache: np.ndarray                 # [num_blocks, Hkv, bs, 2D] float32 (bf16-valued)
    block_table: np.ndarray           # [num_reqs, max_blocks] int
    query_start_loc: np.ndarray       # [num_reqs + 1] int
    seq_lens: np.ndarray              # [num_reqs] int
    scale: float
    staged: dict = field(default_factory=dict)  # request index -> (k_peer, v_peer)
    split_tokens: int = 0
    window: int | None = None         # the impl's sliding_window (ring_backend.py:490-492)


def ring_forward(batch: RingBatch, round_to_bf16: bool = True) -> np.ndarray:
    """Reference ``HcpRingAttentionImpl.forward`` ring path for one layer.

    Restates ``ring_backend.py:597-834`` without the decode-ring branch
    (``:638-727``, a cross-node TCP protocol) and without the debug write
    tracking (``:788-810``):

    * per request: paged gather of all ``tk`` keys (``:616-624``);
    * peer KV = the request's staged segment (``:738-775``) or the first
      ``HCP_RING_SPLIT_TOKENS`` keys of the paged cache (``:776-778``);
    * no peer: plain causal attention at offset ``qpos0`` (``:783-787``);
    * else the ``n_a`` queries still inside the peer region get plain causal
      attention over all keys (``:811-818``) and the rest get local causal
      attention over ``k_all[peer_end:]`` at offset ``qpos0 + n_a - peer_end``
      merged with non-causal attention over the peer KV (``:819-832``);
    * every result is cast to the output dtype (``o.to(output.dtype)``); with
      ``round_to_bf16`` the returned float32 array holds those bf16 values;
    * a sliding window applies to the causal passes only - the vanilla pass,
      the ``n_a`` rows and the local pass - and not to the peer pass
      (``:786, 815, 826`` pass ``self.sliding_window``, ``:829`` does not).

    Returns out [num_tokens, H, D] float32 (rows not covered stay 0).
    """
    q_all = batch.query
    out = np.zeros_like(q_all, dtype=np.float32)
    qsl = [int(x) for x in batch.query_start_loc]
    seq_lens = [int(x) for x in batch.seq_lens]
    cast = round_bf16 if round_to_bf16 else (lambda x: x)
    for r in range(len(seq_lens)):
        qs, qe = qsl[r], qsl[r + 1]
        tq = qe - qs
        tk = seq_lens[r]
        if tq == 0:
            continue
        k_all, v_all = paged_gather(batch.cache, batch.block_table[r], tk)
        staged = batch.staged.get(r)
        plan = plan_request(qs, tq, tk, None if staged is None else staged[0].shape[0],
                            batch.split_tokens)
        q_r = q_all[qs:qe]
        if plan.peer_end == 0:
            o, _ = attn_with_lse(q_r, k_all, v_all, batch.scale, plan.qpos0, batch.window)
            out[qs:qe] = cast(o)
            continue
        if plan.peer_source == "staged":
            k_peer, v_peer = staged
        else:
            k_peer, v_peer = k_all[: plan.peer_end], v_all[: plan.peer_end]
        n_a = plan.n_a
        if n_a > 0:
            o_a, _ = attn_with_lse(q_r[:n_a], k_all, v_all, batch.scale, plan.qpos0, batch.window)
            out[qs:qs + n_a] = cast(o_a)
        if n_a < tq:
            q_b = q_r[n_a:]
            o_loc, lse_loc = attn_with_lse(
                q_b, k_all[plan.peer_end:], v_all[plan.peer_end:], batch.scale,
                plan.qpos0 + n_a - plan.peer_end, batch.window)
            o_peer, lse_peer = attn_with_lse(q_b, k_peer, v_peer, batch.scale, None)
            out[qs + n_a:qe] = cast(lse_merge(o_loc, lse_loc, o_peer, lse_peer))
    return out


# ---------------------------------------------------------------------------
# Decode growth assignment (accumulator ring)
# ---------------------------------------------------------------------------
def merge_chain(states_o, states_lse) -> tuple[np.ndarray, np.ndarray]:
    """Accumulate partials in ring order, as the decode ring's packet does.

    ``states_o`` [N, T, H, D], ``states_lse`` [N, H, T]: the accumulator starts
    as partial 0 and every later partial is merged into it
    (``RingDecodeNode.handle_packet``, ``ring_decode.py:246-247``), each merge
    with :func:`merge_attn_states` (empty partials, lse +/-inf, weigh 0).
    """
    o = np.asarray(states_o[0], np.float32)
    lse = np.asarray(states_lse[0], np.float32)
    for i in range(1, len(states_o)):
        o, lse = merge_attn_states(o, lse, states_o[i], states_lse[i])
    return o, lse


def growth_assignee(pos: int, ring_size: int, policy: str = "rr") -> int:
    """Ring node that keeps the KV of the decode token at global ``pos``.

    Restates ``growth_assignee`` (``hcp_vllm_plugin/ring_decode.py:30-43``):
    ``"owner"`` keeps everything on the owner (index ``ring_size - 1``),
    ``"rr"`` assigns round-robin ``pos % ring_size``.
    """
    if policy == "owner":
        return ring_size - 1
    return pos % ring_size


# ---------------------------------------------------------------------------
# Algorithmic work counts (used by the bench and the roofline)
# ---------------------------------------------------------------------------
def visible_pairs(tq: int, tk: int, causal_offset: int | None) -> int:
    """Number of (query, key) pairs that are not masked out."""
    if causal_offset is None:
        return tq * tk
    total = 0
    # row i sees keys 0 .. min(tk-1, causal_offset + i)
    lo_full = max(0, tk - causal_offset - 1)  # rows i >= lo_full see all tk keys
    for_rows = min(tq, lo_full)
    # rows 0 .. for_rows-1 see causal_offset + i + 1 keys
    total += for_rows * (causal_offset + 1) + for_rows * (for_rows - 1) // 2
    total += (tq - for_rows) * tk
    return total


def attention_flops(pairs: int, num_heads: int, head_dim: int) -> float:
    """4 * D * H FLOPs per visible (query, key) pair (2 for QK^T, 2 for PV)."""
    return 4.0 * head_dim * num_heads * pairs
