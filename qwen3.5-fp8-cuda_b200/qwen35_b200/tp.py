"""Tensor-parallel batch-1 decode over the GPUs of one box.

The decode step shards by heads and by 128-row blocks, with two all-reduces
per layer (the projections shard naturally by output rows; the reference
itself runs on one GPU):

* full attention: rank r owns query heads [h0, h1) and the KV heads they
  read (GQA group g = n_q / n_kv; with more ranks than KV heads two ranks
  compute the same KV head), their KV cache, q_norm/k_norm; o_proj is split
  by its input columns (the rank's heads x head_dim);
* GatedDeltaNet: rank r owns key heads [k0, k1) and value heads
  [2 k0, 2 k1) (32 value heads read key head v // 2): their q/k/v/z/a/b rows,
  conv channels, A_log / dt_bias, recurrent state and conv state; out_proj
  is split by its input columns;
* MLP: gate/up split by output rows in 128-row blocks (SiLU stays local),
  down split by the same columns;
* the column-split projections write FP32 partial sums, all-reduced (sum)
  over the group, then y = bf16(res + bf16(sum)) — the reference's residual
  epilogue applied after the reduction;
* LM head: split by 128-row blocks of the vocabulary; each rank's fused
  argmax packs (orderable BF16 logit << 32 | ~index) with its global row
  offset, the packed keys are all-reduced with MAX (one 8-byte value) and
  the token is decoded from the winner: ties still go to the lowest index.

Embedding, norms and the residual stream are replicated.  The exchanges
run in one of two ways, both captured into the step's CUDA graph:

* ``collective="p2p"`` (default): no library collective.  The column-split
  GEMV stores its FP32 partial rows straight into every rank's exchange
  buffer over NVLink (CUDA IPC mappings, ``qwen_linear_partial_p2p``); the
  residual kernel publishes a flag to every rank, waits (bounded) for every
  rank's flag, sums the slots in rank order and adds the residual
  (``qwen_resid_add_p2p``); the argmax keys go the same way
  (``qwen_token_p2p``).  See csrc/p2p.cuh for the round protocol.
* ``collective="nccl"``: ``torch.distributed.all_reduce`` (SUM of the FP32
  partials, MAX of the packed key) on the engine's stream.

torch.distributed is used for setup in both (the IPC handle exchange).
"""

from __future__ import annotations

import dataclasses

import torch

from . import _lib
from .engine import Qwen35DecodeEngine, _p
from .ops import scale_mode

BLOCK = 128


def _split(n: int, parts: int, r: int) -> tuple[int, int]:
    """Contiguous near-equal split of range(n): part r."""
    base, extra = divmod(n, parts)
    lo = r * base + min(r, extra)
    return lo, lo + base + (1 if r < extra else 0)


@dataclasses.dataclass
class TPLayout:
    rank: int
    world: int
    q_heads: tuple[int, int]      # full-attention query heads
    kv_heads: tuple[int, int]     # full-attention KV heads read by them
    lk_heads: tuple[int, int]     # GatedDeltaNet key heads
    lv_heads: tuple[int, int]     # GatedDeltaNet value heads
    mlp_blocks: tuple[int, int]   # 128-row blocks of the intermediate size
    vocab_blocks: tuple[int, int]  # 128-row blocks of the LM head


def tp_layout(cfg, rank: int, world: int) -> TPLayout:
    """Validate that ``cfg`` shards over ``world`` ranks and return rank's share."""
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    nk, nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
    if nq % world or nk % world or nv % nk or nq % nkv:
        raise ValueError(f"heads ({nq} q, {nk} key, {nv} value) do not split over {world} ranks")
    if cfg.intermediate_size % BLOCK or cfg.vocab_size % BLOCK:
        raise ValueError("intermediate and vocabulary sizes must be multiples of 128")
    if cfg.intermediate_size // BLOCK < world:
        raise ValueError("fewer MLP blocks than ranks")
    g = nq // nkv
    q0, q1 = rank * nq // world, (rank + 1) * nq // world
    kv0, kv1 = q0 // g, (q1 - 1) // g + 1
    k0, k1 = rank * nk // world, (rank + 1) * nk // world
    rep = nv // nk
    return TPLayout(rank, world, (q0, q1), (kv0, kv1), (k0, k1), (k0 * rep, k1 * rep),
                    _split(cfg.intermediate_size // BLOCK, world, rank),
                    _split(cfg.vocab_size // BLOCK, world, rank))


def local_config(cfg, lay: TPLayout):
    """The per-rank model description (local head counts and widths)."""
    return dataclasses.replace(
        cfg,
        num_attention_heads=lay.q_heads[1] - lay.q_heads[0],
        num_key_value_heads=lay.kv_heads[1] - lay.kv_heads[0],
        linear_num_key_heads=lay.lk_heads[1] - lay.lk_heads[0],
        linear_num_value_heads=lay.lv_heads[1] - lay.lv_heads[0],
        intermediate_size=(lay.mlp_blocks[1] - lay.mlp_blocks[0]) * BLOCK,
        layer_types=list(cfg.layer_types))


def _rows(wt, r0: int, r1: int):
    """Rows [r0, r1) of a block-FP8 weight; r0 a multiple of 128 (or the matrix has one scale row)."""
    w, s = wt
    if s.shape[0] == 1:
        return w[r0:r1].contiguous(), s.contiguous()
    assert r0 % BLOCK == 0 and (r1 % BLOCK == 0 or r1 == w.shape[0])
    return w[r0:r1].contiguous(), s[r0 // BLOCK:(r1 + BLOCK - 1) // BLOCK].contiguous()


def _cols(wt, c0: int, c1: int):
    """Input columns [c0, c1) of a block-FP8 weight (multiples of 128)."""
    w, s = wt
    assert c0 % BLOCK == 0 and c1 % BLOCK == 0
    return w[:, c0:c1].contiguous(), s[:, c0 // BLOCK:c1 // BLOCK].contiguous()


def _cat_rows(parts):
    return torch.cat([p[0] for p in parts]).contiguous(), torch.cat([p[1] for p in parts]).contiguous()


def shard_weights(cfg, w: dict, lay: TPLayout) -> dict:
    """This rank's weights (same keys as ``weights.random_weights``)."""
    hd, lkd, lvd = cfg.head_dim, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    (q0, q1), (kv0, kv1) = lay.q_heads, lay.kv_heads
    (k0, k1), (v0, v1) = lay.lk_heads, lay.lv_heads
    m0, m1 = (b * BLOCK for b in lay.mlp_blocks)
    kd = cfg.linear_num_key_heads * lkd
    out = {"embed": w["embed"], "norm_f": w["norm_f"], "layers": []}
    for ly in w["layers"]:
        loc = {"layer_type": ly["layer_type"], "input_layernorm": ly["input_layernorm"],
               "post_attention_layernorm": ly["post_attention_layernorm"]}
        if ly["layer_type"] == "full_attention":
            # q_proj rows are [q | gate] per head (2 * head_dim rows each)
            loc["q_proj"] = _rows(ly["q_proj"], q0 * 2 * hd, q1 * 2 * hd)
            loc["k_proj"] = _rows(ly["k_proj"], kv0 * hd, kv1 * hd)
            loc["v_proj"] = _rows(ly["v_proj"], kv0 * hd, kv1 * hd)
            loc["o_proj"] = _cols(ly["o_proj"], q0 * hd, q1 * hd)
            loc["q_norm"], loc["k_norm"] = ly["q_norm"], ly["k_norm"]
        else:
            qkv = ly["in_proj_qkv"]
            loc["in_proj_qkv"] = _cat_rows([_rows(qkv, k0 * lkd, k1 * lkd),
                                            _rows(qkv, kd + k0 * lkd, kd + k1 * lkd),
                                            _rows(qkv, 2 * kd + v0 * lvd, 2 * kd + v1 * lvd)])
            cw = ly["conv1d_w"]
            loc["conv1d_w"] = torch.cat([cw[k0 * lkd:k1 * lkd], cw[kd + k0 * lkd:kd + k1 * lkd],
                                         cw[2 * kd + v0 * lvd:2 * kd + v1 * lvd]]).contiguous()
            loc["in_proj_z"] = _rows(ly["in_proj_z"], v0 * lvd, v1 * lvd)
            loc["in_proj_a"] = _rows(ly["in_proj_a"], v0, v1)
            loc["in_proj_b"] = _rows(ly["in_proj_b"], v0, v1)
            loc["A_log"] = ly["A_log"][v0:v1].contiguous()
            loc["dt_bias"] = ly["dt_bias"][v0:v1].contiguous()
            loc["norm_w"] = ly["norm_w"]
            loc["out_proj"] = _cols(ly["out_proj"], v0 * lvd, v1 * lvd)
        loc["gate_proj"] = _rows(ly["gate_proj"], m0, m1)
        loc["up_proj"] = _rows(ly["up_proj"], m0, m1)
        loc["down_proj"] = _cols(ly["down_proj"], m0, m1)
        out["layers"].append(loc)
    head = w["lm_head"]
    if not isinstance(head, tuple):
        raise NotImplementedError("tensor parallelism needs the block-FP8 LM head")
    out["lm_head"] = _rows(head, lay.vocab_blocks[0] * BLOCK, lay.vocab_blocks[1] * BLOCK)
    out["lm_row_offset"] = lay.vocab_blocks[0] * BLOCK
    return out


class Qwen35TPDecodeEngine(Qwen35DecodeEngine):
    """One rank of the tensor-parallel greedy decoder.

    Every rank is driven with the same tokens (the residual stream, position
    and greedy token are replicated); ``group`` is an initialised process
    group of ``world`` ranks, one GPU each (NCCL for ``collective="nccl"``).
    """

    def __init__(self, cfg, weights, rank: int, world: int, group=None, collective: str = "p2p", **kw):
        import torch.distributed as dist
        if collective not in ("p2p", "nccl"):
            raise ValueError(f"collective must be 'p2p' or 'nccl', not {collective!r}")
        self.full_cfg = cfg
        self.layout = tp_layout(cfg, rank, world)
        self.dist = dist
        self.group = group
        self.collective = collective
        self.rank, self.world = rank, world
        lcfg = local_config(cfg, self.layout)
        lw = shard_weights(cfg, weights, self.layout)
        super().__init__(lcfg, lw, **kw)
        self.partial = torch.zeros(cfg.hidden_size, dtype=torch.float32, device=self.device)
        self._p2p_base = self._p2p_table = None
        self._p2p_peers = []
        if collective == "p2p":
            self._p2p_setup(cfg.hidden_size)
        # launches per decoder layer in the plan (the layer-by-layer tests step
        # through them); with p2p a layer's output stream is written by the
        # next layer's first launch (or the LM head)
        self.launches_per_layer = 5 if collective == "p2p" else 9

    def _p2p_setup(self, n: int):
        """Allocate this rank's exchange region, map every peer's (CUDA IPC)
        and build the device table."""
        import ctypes
        lib, dist = self.lib, self.dist
        base = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(lib.qwen_p2p_create(self.world, n, ctypes.byref(base), handle), "qwen_p2p_create")
        self._p2p_base = base
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        bases = []
        for r in range(self.world):
            if r == self.rank:
                bases.append(base.value)
                continue
            pb = ctypes.c_void_p()
            _lib.check(lib.qwen_p2p_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(pb)),
                       "qwen_p2p_open")
            self._p2p_peers.append(pb)
            bases.append(pb.value)
        arr = (ctypes.c_void_p * self.world)(*bases)
        table = ctypes.c_void_p()
        _lib.check(lib.qwen_p2p_table(arr, self.world, self.rank, n, ctypes.byref(table)), "qwen_p2p_table")
        self._p2p_table = table
        dist.barrier(group=self.group)

    def close(self):
        """Release the step graphs (with NCCL exchanges they hold NCCL calls,
        which must go before the process group is destroyed), then unmap the
        peers' exchange regions and free this rank's (collective: every rank
        calls it, after its last step)."""
        torch.cuda.synchronize(self.device)
        self.graph = None
        self.graph_io = None
        if self._p2p_base is None:
            return
        self.dist.barrier(group=self.group)
        for pb in self._p2p_peers:
            self.lib.qwen_p2p_close(pb)
        self.lib.qwen_p2p_table_free(self._p2p_table)
        self.lib.qwen_p2p_destroy(self._p2p_base)
        self._p2p_base = self._p2p_table = None
        self._p2p_peers = []

    def _plan_step(self):
        cfg, lib, w, dist = self.cfg, self.lib, self.w, self.dist
        H, I = cfg.hidden_size, cfg.intermediate_size
        eps = cfg.rms_norm_eps
        plan = []

        def chk(status, what):
            _lib.check(status, what)

        def allreduce_sum(st):
            dist.all_reduce(self.partial, op=dist.ReduceOp.SUM, group=self.group)

        p2p = self.collective == "p2p"
        table = self._p2p_table
        # p2p: the launch after a partial GEMV (gate/up, the next in_proj or
        # the LM head) takes its input from the exchange plus the residual:
        # no separate reduction launch
        pending = []

        def add(launch, regions):
            if pending:
                res = pending.pop()
                inner = launch

                def launch(st, inner=inner, res=res):
                    chk(lib.qwen_set_p2p_input(table, _p(res), H), "p2p_input")
                    return inner(st)
            plan.append((launch, regions))

        def partial_resid(x, wt, res, out, gated=None):
            """gated = (z, norm_w): x is a GatedDeltaNet core output whose gated
            norm runs in this GEMV's prologue."""
            wo, so = wt

            def pre():
                if gated is not None:
                    chk(lib.qwen_set_gated_input(_p(gated[0]), _p(gated[1]), eps), "gated_input")
            if p2p:
                plan.append((lambda st: (pre(), chk(lib.qwen_linear_partial_p2p(
                    _p(x), _p(wo), _p(so), wo.shape[0], wo.shape[1], scale_mode(wo.shape[0], so), table, st),
                    "linear_partial_p2p")), self._regions(wo)))
                pending.append(res)  # the consumer writes bf16(res + sum) to `out`, its x
                return
            plan.append((lambda st: (pre(), chk(lib.qwen_linear_partial(
                _p(x), _p(wo), _p(so), wo.shape[0], wo.shape[1], scale_mode(wo.shape[0], so),
                _p(self.partial), st), "linear_partial")), self._regions(wo)))
            plan.append((allreduce_sum, []))
            plan.append((lambda st: chk(lib.qwen_resid_add_f32(_p(res), _p(self.partial), _p(out), H, st),
                                        "resid_add"), []))

        plan.append((lambda st: chk(lib.qwen_embed(_p(w["embed"]), _p(self.token), _p(self.hidden), H, st),
                                    "qwen_embed"), []))
        for i, ly in enumerate(w["layers"]):
            if cfg.layer_types[i] == "full_attention":
                (wq, sq), (wk, sk), (wv, sv) = ly["q_proj"], ly["k_proj"], ly["v_proj"]
                add(lambda st, ly=ly, wq=wq, sq=sq, wk=wk, sk=sk, wv=wv, sv=sv: chk(lib.qwen_attn_in_proj(
                    _p(self.hidden), _p(ly["input_layernorm"]), eps, _p(wq), _p(sq), wq.shape[0], _p(wk), _p(sk),
                    wk.shape[0], _p(wv), _p(sv), wv.shape[0], H, scale_mode(wq.shape[0], sq), _p(self.q_all),
                    _p(self.k_new), _p(self.v_new), st), "attn_in_proj"), self._regions(wq, wk, wv))
                plan.append((lambda st, ly=ly, i=i: chk(lib.qwen_attn_decode(
                    _p(self.q_all), _p(self.k_new), _p(self.v_new), _p(ly["q_norm"]), _p(ly["k_norm"]),
                    _p(self.cos), _p(self.sin), _p(self.k_cache[i]), _p(self.v_cache[i]), _p(self.pos),
                    self.max_seq, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rotary_dim, eps,
                    self.attn_chunk, self.attn_nsplit, _p(self.attn_ws), _p(self.attn_cnt), _p(self.attn_out), st),
                    "attn_decode"), []))
                partial_resid(self.attn_out, ly["o_proj"], self.hidden, self.h2)
            else:
                (wqkv, sqkv), (wz, sz) = ly["in_proj_qkv"], ly["in_proj_z"]
                (wa, sa), (wb, sb) = ly["in_proj_a"], ly["in_proj_b"]
                add(lambda st, ly=ly, i=i, wqkv=wqkv, sqkv=sqkv, wz=wz, sz=sz, wa=wa, sa=sa, wb=wb, sb=sb:
                             chk(lib.qwen_gdn_in_proj(
                                 _p(self.hidden), _p(ly["input_layernorm"]), eps, H, scale_mode(wqkv.shape[0], sqkv),
                                 _p(wqkv), _p(sqkv), wqkv.shape[0], _p(ly["conv1d_w"]), _p(self.conv_state[i]),
                                 cfg.linear_conv_kernel_dim, _p(self.qkv_conv), _p(wz), _p(sz), wz.shape[0],
                                 _p(self.z), _p(wa), _p(sa), _p(wb), _p(sb), wa.shape[0], _p(ly["A_log"]),
                                 _p(ly["dt_bias"]), _p(self.g), _p(self.beta), st), "gdn_in_proj"),
                             self._regions(wqkv, wz, wa, wb))
                if self.gdn_split:
                    plan.append((lambda st, i=i: chk(lib.qwen_gdn_decode_core(
                        _p(self.qkv_conv), _p(self.g), _p(self.beta), _p(self.state[i]), _p(self.attn_out),
                        cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_value_head_dim, st),
                        "gdn_decode_core"), []))
                    partial_resid(self.attn_out, ly["out_proj"], self.hidden, self.h2,
                                  gated=(self.z, ly["norm_w"]))
                else:
                    plan.append((lambda st, ly=ly, i=i: chk(lib.qwen_gdn_decode(
                        _p(self.qkv_conv), _p(self.g), _p(self.beta), _p(self.state[i]), _p(self.z),
                        _p(ly["norm_w"]), eps, _p(self.attn_out), cfg.linear_num_key_heads,
                        cfg.linear_num_value_heads, cfg.linear_value_head_dim, st), "gdn_decode"), []))
                    partial_resid(self.attn_out, ly["out_proj"], self.hidden, self.h2)
            (wg, sg), (wu, su) = ly["gate_proj"], ly["up_proj"]
            add(lambda st, ly=ly, wg=wg, sg=sg, wu=wu, su=su: chk(lib.qwen_mlp_gate_up(
                _p(self.h2), _p(ly["post_attention_layernorm"]), eps, _p(wg), _p(sg), _p(wu), _p(su), I, H,
                scale_mode(I, sg), _p(self.silu), st), "gate_up"), self._regions(wg, wu))
            partial_resid(self.silu, ly["down_proj"], self.h2, self.hidden)
        wh, sh = w["lm_head"]
        add(lambda st: chk(lib.launch_lm_head_argmax(
            _p(self.hidden), _p(w["norm_f"]), eps, _p(wh), _p(sh), wh.shape[0], H, scale_mode(wh.shape[0], sh),
            w["lm_row_offset"], _p(self.am_ws), _p(self.key), _p(self.token), _p(self.logits), _p(self.pos), st),
            "lm_head_argmax"), self._regions(wh))
        if p2p:
            plan.append((lambda st: chk(lib.qwen_token_p2p(table, _p(self.key), _p(self.token), st), "token_p2p"),
                         []))
            self.collectives_per_step = 0
            return plan
        plan.append((lambda st: dist.all_reduce(self.key, op=dist.ReduceOp.MAX, group=self.group), []))
        plan.append((lambda st: chk(lib.qwen_token_from_key(_p(self.key), _p(self.token), st), "token"), []))
        self.collectives_per_step = sum(1 for f, _ in plan if f is allreduce_sum) + 1
        return plan

    def _mutable(self):
        return super()._mutable() + [self.partial]
