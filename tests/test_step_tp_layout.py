"""Host logic of the tensor-parallel step engine (qwen35_b200/step_tp.py), on CPU.

The stage lists of every rank are built against synthetic device addresses
(one 2^40-byte window per matrix or buffer) and checked:

* every column-parallel matrix (in_proj / q / k / v, gate/up, LM head) has
  each output row computed by exactly one rank (the per-head gate rows
  a / b by every rank; with more ranks than KV heads, q / k / v rows of a head
  by the ranks sharing it), and every segment's packed weights, outputs and
  per-row epilogue operands stay inside their allocations;
* every row-parallel matrix (out_proj, o_proj, down) has its K chunks split
  into contiguous ranges in rank order whose union is K, x read inside its
  buffer at the range's offset, and cstride = the whole matrix's K / 512;
* GatedDeltaNet / attention shards cover the heads whose rows the rank's
  in_proj / q, k, v segments computed, and the o_proj / out_proj K range
  reads only heads the rank's mixer wrote;
* slice producers alternate between the two K-slice buffers, and every
  reader of a buffer follows its producer.
"""

import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "qwen3.5-fp8-cuda_b200"))

from qwen35_b200.config import qwen35_4b, qwen35_tiny  # noqa: E402
from qwen35_b200.step import (ATTN, EPI_ARGMAX, EPI_CONV, EPI_GATE_BETA, EPI_GATE_G, EPI_SILU,  # noqa: E402
                              EPI_SILU_PAIR, EPI_SLICES, EPI_STORE, GDN, GEMV, PRO_SLICES_NORM)
from qwen35_b200.step_tp import CHUNK_BYTES, CHUNK_K, TILE_ROWS, Qwen35StepTPEngine  # noqa: E402

WIN = 1 << 40


class _T:
    """A stand-in tensor: a shape and a synthetic device address."""

    def __init__(self, space, name, shape, esize):
        self.shape, self.esize, self.name = tuple(shape), esize, name
        n = 1
        for d in shape:
            n *= d
        self.nbytes = n * esize
        self.addr = space.add(name, self.nbytes)

    def data_ptr(self):
        return self.addr


class _Space:
    def __init__(self):
        self.allocs = []

    def add(self, name, nbytes):
        self.allocs.append((name, nbytes))
        return len(self.allocs) * WIN

    def where(self, addr):
        i = addr // WIN - 1
        assert 0 <= i < len(self.allocs), hex(addr)
        return self.allocs[i][0], addr % WIN, self.allocs[i][1]


def _packed_bytes(n, k, bf16=False):
    return (n + TILE_ROWS - 1) // TILE_ROWS * (k // (256 if bf16 else CHUNK_K)) * CHUNK_BYTES


def _fake_engine(cfg, rank, world, bf16_head=False):
    sp = _Space()
    e = Qwen35StepTPEngine.__new__(Qwen35StepTPEngine)
    e.cfg, e.rank, e.world, e.nslice = cfg, rank, world, 1
    e.max_seq, e.attn_chunk, e.attn_nsplit = 64, 16, 4
    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    e.packed = {}

    def mat(name, n, k):
        w = _T(sp, name, (n, k), 1)
        e.packed[w.addr] = _T(sp, name + ".packed", (_packed_bytes(n, k),), 1)
        return (w, _T(sp, name + ".scale", ((n + 127) // 128, k // 128), 4))

    def vec(name, n, esize=2):
        return _T(sp, name, (n,), esize)

    if bf16_head:
        head = _T(sp, "lm_head", (V, H), 2)
        e.packed[head.addr] = _T(sp, "lm_head.packed", (_packed_bytes(V, H, True),), 1)
    else:
        head = mat("lm_head", V, H)
    layers = []
    cw = cfg.linear_conv_kernel_dim
    for i in range(cfg.num_hidden_layers):
        ly = dict(input_layernorm=vec(f"{i}.ln1", H, 4), post_attention_layernorm=vec(f"{i}.ln2", H, 4),
                  gate_proj=mat(f"{i}.gate", I, H), up_proj=mat(f"{i}.up", I, H), down_proj=mat(f"{i}.down", H, I))
        if cfg.layer_types[i] == "full_attention":
            ly.update(q_proj=mat(f"{i}.q", nh * hd * 2, H), k_proj=mat(f"{i}.k", nkv * hd, H),
                      v_proj=mat(f"{i}.v", nkv * hd, H), o_proj=mat(f"{i}.o", H, nh * hd),
                      q_norm=vec(f"{i}.qn", hd, 4), k_norm=vec(f"{i}.kn", hd, 4))
        else:
            nv = cfg.linear_num_value_heads
            ly.update(in_proj_qkv=mat(f"{i}.qkv", cfg.conv_dim, H), in_proj_z=mat(f"{i}.z", cfg.linear_value_dim, H),
                      in_proj_a=mat(f"{i}.a", nv, H), in_proj_b=mat(f"{i}.b", nv, H),
                      out_proj=mat(f"{i}.out", H, cfg.linear_value_dim),
                      conv1d_w=_T(sp, f"{i}.conv_w", (cfg.conv_dim, cw), 2), A_log=vec(f"{i}.A_log", nv, 4),
                      dt_bias=vec(f"{i}.dt_bias", nv, 4), norm_w=vec(f"{i}.gnorm", cfg.linear_value_head_dim, 4))
        layers.append(ly)
    e.w = dict(embed=_T(sp, "embed", (V, H), 2), norm_f=vec("norm_f", H, 4), lm_head=head, layers=layers)
    qd = nh * hd
    e.q_all, e.k_new, e.v_new = vec("q_all", 2 * qd), vec("k_new", nkv * hd), vec("v_new", nkv * hd)
    e.attn_out = vec("attn_out", max(qd, cfg.linear_value_dim))
    e.qkv_conv, e.z = vec("qkv_conv", cfg.conv_dim), vec("z", cfg.linear_value_dim)
    e.g, e.beta = vec("g", cfg.linear_num_value_heads, 4), vec("beta", cfg.linear_num_value_heads)
    e.silu, e.hidden, e.h2 = vec("silu", I), vec("hidden", H), vec("h2", H)
    e.sl_buf, e.sl_buf2 = vec("sl_buf", 16 * H, 4), vec("sl_buf2", 16 * H, 4)
    e.logits, e.token, e.key = vec("logits", V), vec("token", 1, 8), vec("key", 1, 8)
    e.pos, e.am_ws = vec("pos", 1, 4), vec("am_ws", 2, 8)
    e.cos, e.sin = vec("cos", 64 * hd, 4), vec("sin", 64 * hd, 4)
    e.attn_ws, e.attn_cnt = vec("attn_ws", 1 << 20, 4), vec("attn_cnt", nkv, 4)
    e.k_cache, e.v_cache, e.state, e.conv_state = {}, {}, {}, {}
    for i in range(cfg.num_hidden_layers):
        if cfg.layer_types[i] == "full_attention":
            e.k_cache[i], e.v_cache[i] = vec(f"{i}.kc", 64 * qd), vec(f"{i}.vc", 64 * qd)
        else:
            e.state[i] = vec(f"{i}.state", 1 << 20, 4)
            e.conv_state[i] = _T(sp, f"{i}.conv_state", (cfg.conv_dim, cw), 2)
    return e, sp


def _in(sp, addr, nbytes, name):
    n, off, size = sp.where(addr)
    assert n == name, (n, name)
    assert 0 <= off and off + nbytes <= size, (name, off, nbytes, size)
    return off


def _tp_cfg():
    # the small member widened so every split stays 512-aligned up to 4 ranks
    return qwen35_tiny(intermediate_size=4096, num_attention_heads=8, num_key_value_heads=2,
                       linear_num_key_heads=8, linear_num_value_heads=16)


@pytest.mark.parametrize("cfg_name,world,bf16_head", [("tp_tiny", 2, False), ("tp_tiny", 4, False),
                                                      ("4b", 2, False), ("4b", 4, False), ("4b", 8, False),
                                                      ("4b", 8, True)])
def test_tp_stage_split(cfg_name, world, bf16_head):
    cfg = _tp_cfg() if cfg_name == "tp_tiny" else qwen35_4b()
    H = cfg.hidden_size
    rows = {}    # matrix name -> per-row count of ranks computing it
    kparts = {}  # row-parallel matrix name -> [(rank, c0, c1)]
    for rank in range(world):
        e, sp = _fake_engine(cfg, rank, world, bf16_head)
        stages = list(e._build_stages())
        assert len(stages) == 5 * cfg.num_hidden_layers + 1
        last_sl = None
        gdn_heads = attn_kv = None
        for si, st in enumerate(stages):
            if st.kind == GEMV:
                if st.pro == PRO_SLICES_NORM:  # reads the buffer the latest slice producer wrote
                    assert st.sl_in == last_sl and st.sl_stride == H
                for j in range(st.nseg):
                    sg = st.seg[j]
                    wname, woff, _ = sp.where(sg.w)
                    mname = wname[:-len(".packed")]
                    if sg.epi == EPI_SLICES:  # row-parallel
                        assert st.nseg == 1 and st.xrank == 1
                        C = st.cstride
                        assert woff % CHUNK_BYTES == 0 and st.K % CHUNK_K == 0
                        c0 = woff // CHUNK_BYTES
                        c1 = c0 + st.K // CHUNK_K
                        _in(sp, sg.w, (((sg.n + 31) // 32 - 1) * C + c1 - c0) * CHUNK_BYTES, wname)
                        xname, xoff, _ = sp.where(st.x)
                        assert xoff == 2 * c0 * CHUNK_K
                        _in(sp, st.x, 2 * st.K, xname)
                        kparts.setdefault(mname, []).append((rank, c0, c1, C))
                        # the mixer wrote the heads this K range reads
                        if mname.endswith(".out"):
                            dv = cfg.linear_value_head_dim
                            assert gdn_heads[0] * dv == c0 * CHUNK_K and gdn_heads[1] * dv == c1 * CHUNK_K
                        elif mname.endswith(".o"):
                            G = cfg.num_attention_heads // cfg.num_key_value_heads
                            lo, hi = c0 * CHUNK_K // cfg.head_dim, c1 * CHUNK_K // cfg.head_dim
                            assert attn_kv[0] * G <= lo and hi <= attn_kv[1] * G
                        assert sg.n == H and st.sl_rows == H
                        last_sl = st.sl_out
                        assert sp.where(last_sl)[0] == ("sl_buf2" if mname.endswith(".down") else "sl_buf")
                        continue
                    bf = bool(st.wbf16)
                    C = st.K // (256 if bf else CHUNK_K)
                    assert woff % (C * CHUNK_BYTES) == 0
                    r0 = woff // (C * CHUNK_BYTES) * TILE_ROWS
                    _in(sp, sg.w, (sg.n + 31) // 32 * C * CHUNK_BYTES, wname)
                    if st.pair:
                        _in(sp, sg.w2, (sg.n + 31) // 32 * C * CHUNK_BYTES, sp.where(sg.w2)[0])
                        assert sp.where(sg.w2)[1] == woff
                    esize = 4 if sg.epi == EPI_GATE_G else 2
                    if sg.y:
                        yname, yoff, _ = sp.where(sg.y)
                        _in(sp, sg.y, esize * sg.n, yname)
                    if sg.epi == EPI_CONV:
                        # rows of in_proj_qkv = conv channels: output, weights and state at the same row
                        assert yoff == 2 * r0
                        assert sp.where(sg.aux0)[1] == 2 * r0 * sg.cw
                        assert sp.where(sg.aux2)[1] == 2 * r0 * sg.cw
                        _in(sp, sg.aux2, 2 * sg.n * sg.cw, sp.where(sg.aux2)[0])
                    elif sg.epi == EPI_GATE_G:
                        assert yoff == 4 * r0 and sp.where(sg.aux0)[1] == 4 * r0
                    elif sg.epi == EPI_ARGMAX:
                        assert sg.row_offset == r0 and (not sg.y or yoff == 2 * r0)
                    elif sg.epi in (EPI_STORE, EPI_SILU_PAIR, EPI_GATE_BETA, EPI_SILU):
                        assert yoff == 2 * r0
                    cnt = rows.setdefault(mname, {})
                    for r in range(r0, r0 + sg.n):
                        cnt[r] = cnt.get(r, 0) + 1
            elif st.kind == GDN:
                gdn_heads = (st.shard0, st.shard0 + st.shard_n)
                assert st.shard_n > 0
                # the rank's in_proj wrote these heads' q / k / v / z rows
                prev = stages[si - 1]
                dv, dk = cfg.linear_value_head_dim, cfg.linear_key_head_dim
                zs = [prev.seg[j] for j in range(prev.nseg) if sp.where(prev.seg[j].y)[0] == "z"][0]
                assert sp.where(zs.y)[1] == 2 * gdn_heads[0] * dv and zs.n == st.shard_n * dv
                rep = cfg.linear_num_value_heads // cfg.linear_num_key_heads
                qs = prev.seg[0]
                assert sp.where(qs.y)[1] == 2 * (gdn_heads[0] // rep) * dk
            elif st.kind == ATTN:
                attn_kv = (st.shard0, st.shard0 + st.shard_n)
                assert st.shard_n > 0
                prev = stages[si - 1]
                hd = cfg.head_dim
                assert sp.where(prev.seg[1].y)[1] == 2 * attn_kv[0] * hd and prev.seg[1].n == st.shard_n * hd
    # column-parallel coverage
    nkv = cfg.num_key_value_heads
    dup = max(1, world // nkv)
    for name, cnt in rows.items():
        n = {"lm_head": cfg.vocab_size}.get(name)
        layer, kind = (name.split(".") + [""])[:2] if name != "lm_head" else ("", "lm_head")
        want = 1
        if kind in ("a", "b"):
            want = world
        elif kind in ("q", "k", "v"):
            want = dup
        if n is None:
            n = max(cnt) + 1
        assert sorted(cnt) == list(range(n)), name
        assert set(cnt.values()) == {want}, (name, set(cnt.values()), want)
    # every in_proj row of every linear layer, every MLP intermediate row
    for i in range(cfg.num_hidden_layers):
        assert len(rows[f"{i}.gate"]) == cfg.intermediate_size
        if cfg.layer_types[i] != "full_attention":
            assert len(rows[f"{i}.qkv"]) == cfg.conv_dim and len(rows[f"{i}.z"]) == cfg.linear_value_dim
    assert len(rows["lm_head"]) == cfg.vocab_size
    # row-parallel: contiguous K ranges in rank order covering K
    for name, parts in kparts.items():
        parts.sort()
        assert [p[0] for p in parts] == list(range(world)), name
        C = parts[0][3]
        assert parts[0][1] == 0 and parts[-1][2] == C, name
        for a, b in zip(parts, parts[1:]):
            assert a[2] == b[1], name


def test_tp_split_rejects_unaligned():
    cfg = qwen35_tiny()  # 4 value heads x 128: out_proj K = 512 cannot be split over 2 ranks
    e, _ = _fake_engine(cfg, 0, 2)
    with pytest.raises(ValueError):
        e._build_stages()
