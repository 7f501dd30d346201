"""Generate the golden fixtures by running the REFERENCE's own torch code on the inputs of cases.py.

Usage (needs the reference checkout, read-only):
    python tests/golden/gen_golden.py --reference /path/to/hybrid-latent-attention [--only step_context]
    (or set HLA_REFERENCE_ROOT instead of passing --reference)

Writes tests/golden/<name>.npz with the reference outputs and a sha256 of the inputs.
The reference functions called (file:line in the reference project):
  hla/vllm_latent/s6_ops.py:117 history_attention (torch backend -> _history_reference :204)
  hla/vllm_latent/s6_ops.py:290 window_attention, :234 chunk_attention('torch'), :353 merge_lse
  hla/vllm_latent/s6_ops.py:262 merge_states('torch'), :23 latent_rope('torch'), :61 token_requests,
  :71 history_lengths, :76 num_kv_splits
  hla/vllm_latent/s6_layer.py:43 StepContext (the integer fields and block_table; step_context.json)
  hla/vllm_latent/s6_layer.py:16 latent_inv_freq, :21 latent_rope_table, :32 latent_query,
  :124 write_rows, :135 committed_row
  hla/latent/register.py:28 LatentLayer (write_step / write1 / pack / fields)
  hla/latent/fused_history.py:11 reference (the contiguous-layout reader's torch definition)
  hla/vllm_latent/cache_export.py:13 RolloutCacheExporter (begin / observe / export / finish), driven
  through a stand-in runner that exposes the attributes the exporter reads
  BASELINE config 1 (config1.npz): s6_layer.latent_query('torch', bf16 table) per loop, then in fp32
  s6_ops.history_attention('torch'), the B einsum (s6_layer.py:114), chunk_attention('torch') over the
  current token + window_attention + merge_lse (the exact window), and merge_states('torch')
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def step_context_fixture(s6_layer, s6_ops, torch):
    """Integer fields of the reference's StepContext (s6_layer.py:52-77) on cases.step_context_cases()."""
    rows = []
    for qsl, seq_lens, T, window, table in cases.step_context_cases():
        ctx = s6_layer.StepContext(torch.zeros(T, dtype=torch.long), torch.tensor(qsl, dtype=torch.int32),
                                   torch.tensor(seq_lens, dtype=torch.int32), 1, T, {}, 1.0,
                                   s6_ops.TORCH_BACKENDS, window=window)
        rows.append(dict(token_requests=ctx.token_requests.tolist(), valid=ctx.valid.tolist(),
                         invalid=ctx.invalid.tolist(), ctx=ctx.ctx.tolist(), ctx_latent=ctx.ctx_latent.tolist(),
                         empty=ctx.empty.tolist(), empty_latent=ctx.empty_latent.tolist(),
                         ctx_dtype=str(ctx.ctx.dtype), ctx_latent_dtype=str(ctx.ctx_latent.dtype),
                         block_table=ctx.block_table(torch.tensor(table, dtype=torch.int32)).tolist()))
    (HERE / 'step_context.json').write_text(json.dumps(rows))
    print('wrote step_context.json', len(rows))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default=os.environ.get('HLA_REFERENCE_ROOT'),
                    help='checkout of the reference project (default: $HLA_REFERENCE_ROOT)')
    ap.add_argument('--only', choices=['step_context'], help='write only this fixture')
    args = ap.parse_args()
    if not args.reference:
        ap.error('pass --reference or set HLA_REFERENCE_ROOT to a checkout of the reference project')
    sys.path.insert(0, args.reference)
    import torch
    from hla.latent.register import LatentLayer
    from hla.vllm_latent import s6_layer, s6_ops
    torch.set_num_threads(4)
    T_ = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    step_context_fixture(s6_layer, s6_ops, torch)
    if args.only:
        return

    def save(name, inputs, **outputs):
        np.savez_compressed(HERE / f'{name}.npz', input_sha256=np.array(cases.digest(inputs)), **outputs)
        print('wrote', name, {k: getattr(v, 'shape', v) for k, v in outputs.items()})

    # ---- A1 history reader
    for name, (inp, scale) in cases.history_cases().items():
        o, lse = s6_ops.history_attention(T_(inp['q']), T_(inp['cache']), T_(inp['block_table']), T_(inp['ctx']),
                                          float(scale), 1, None, None, None, 'torch')
        save(name, inp, o=o.numpy(), lse=lse.numpy(), scale=np.float64(scale))

    # ---- A5 decode window (the reference's own non-fused composition of the same keys as
    #      window_attention_fa: chunk over the current token + window history + merge_lse)
    w = cases.window_case()
    q, phys, table = T_(w['q']), T_(w['cache_phys']), T_(w['block_table'])
    qsl, seq_lens, window = T_(w['query_start_loc']), T_(w['seq_lens']), int(w['window'])
    Tn, H, d = q.shape
    page = phys.shape[1]
    logical = phys.transpose(1, 2)                       # [nb, H, page, 2d]
    req, valid = s6_ops.token_requests(qsl, Tn)
    invalid = ~valid
    last = (seq_lens[req] - 1).clamp(min=0)
    blk = table[req, last // page].long()
    cur = phys[blk, last % page]                          # [T, H, 2d] current token rows
    k_cur, v_cur = cur[..., :d].contiguous(), cur[..., d:].contiguous()
    scale = 1 / math.sqrt(d)
    o_c, lse_c = s6_ops.chunk_attention(q, k_cur, v_cur, torch.arange(Tn + 1, dtype=torch.int32).clamp(max=int(qsl[-1])),
                                        1, invalid, scale, 'torch')
    ctx = torch.where(valid, last, 0).int()
    o_w, lse_w = s6_ops.window_attention(q, logical, table[req], ctx, window, scale)
    o, lse = s6_ops.merge_lse(o_w, lse_w, o_c, lse_c)
    o = o.masked_fill(invalid[:, None, None], 0)
    lse = lse.masked_fill(invalid[None, :], -float('inf'))
    save('window_decode', w, o=o.numpy(), lse=lse.numpy(), scale=np.float64(scale))

    # ---- one layer x 4 loops of the decode op in fp32 (latent query with the bf16 table
    #      as serving computes it, then history + B + exact window + merge with fp32 arithmetic)
    c1 = cases.config1_case()
    inv = s6_layer.latent_inv_freq(128, float(c1['latent_theta']))
    tabs = {w: s6_layer.latent_rope_table(int(c1['max_pos']), inv, w, torch.bfloat16) for w in (256, 512)}
    pos = T_(c1['positions'])
    qsl, seq_lens, table = T_(c1['query_start_loc']), T_(c1['seq_lens']), T_(c1['table'])
    ctx1, ctx_lat1, window = T_(c1['ctx']), T_(c1['ctx_lat']), int(c1['window'])
    scale = 1 / math.sqrt(128)
    invalid = torch.zeros(1, dtype=torch.bool)
    outs = {}
    for t in range(4):
        w = 256 if t == 0 else 512
        q_lat = s6_layer.latent_query(T_(c1[f'q_pre{t}']).bfloat16(), T_(c1[f'A{t}']).bfloat16(), pos, tabs[w], 'torch')
        q_lat = q_lat.float()
        cache = T_(c1['lat_l1'] if t == 0 else c1['lat_main'])
        o_h, lse_h = s6_ops.history_attention(q_lat, cache, table, ctx_lat1, scale, 1, None, None, None, 'torch')
        o_h = torch.einsum('thr,hrd->thd', o_h, T_(c1[f'B{t}']))
        phys = T_(c1[f'exact{t}'])
        last = int(c1['ctx'][0])
        cur = phys[int(c1['table'][0, last // 16]), last % 16][None]          # [1, H, 2d]
        q_rope = T_(c1[f'q_rope{t}'])
        o_c, lse_c = s6_ops.chunk_attention(q_rope, cur[..., :128].contiguous(), cur[..., 128:].contiguous(), qsl, 1,
                                            invalid, scale, 'torch')
        o_w, lse_w = s6_ops.window_attention(q_rope, phys.transpose(1, 2), table, ctx1, window, scale)
        o_x, lse_x = s6_ops.merge_lse(o_w, lse_w, o_c, lse_c)
        out = s6_ops.merge_states(o_h, lse_h, o_x, lse_x, invalid, 'torch')
        outs[f'q_lat{t}'] = q_lat.numpy()
        outs[f'lse_hist{t}'] = lse_h.numpy()
        outs[f'out{t}'] = out.numpy()
    save('config1', c1, scale=np.float64(scale), **outs)

    # ---- A5 prefill pieces: causal chunk attention and the per-token window history
    c = cases.chunk_case()
    qsl = T_(c['query_start_loc'])
    n = int(c['num_tokens'])
    _, valid = s6_ops.token_requests(qsl, n)
    o, lse = s6_ops.chunk_attention(T_(c['q']), T_(c['k']), T_(c['v']), qsl, 41, ~valid, 1 / math.sqrt(128), 'torch')
    save('chunk', c, o=o.numpy(), lse=lse.numpy(), scale=np.float64(1 / math.sqrt(128)))
    wh = cases.window_history_case()
    logical = T_(wh['cache_phys']).transpose(1, 2)
    o, lse = s6_ops.window_attention(T_(wh['q']), logical, T_(wh['block_table']), T_(wh['ctx']), int(wh['window']),
                                     1 / math.sqrt(128))
    save('window_history', wh, o=o.numpy(), lse=lse.numpy(), scale=np.float64(1 / math.sqrt(128)))

    # ---- A7 merges
    m = cases.merge_case()
    out = s6_ops.merge_states(T_(m['o_hist']), T_(m['lse_hist']), T_(m['o_chunk']), T_(m['lse_chunk']),
                              T_(m['invalid']), 'torch')
    l_c_noinf = np.where(m['lse_chunk'] == np.inf, -np.inf, m['lse_chunk']).astype(np.float32)
    o2, l2 = s6_ops.merge_lse(T_(m['o_hist']), T_(m['lse_hist']), T_(m['o_chunk']), T_(l_c_noinf))
    save('merge', m, merge_states=out.numpy(), merge_lse_o=o2.numpy(), merge_lse_lse=l2.numpy())

    # ---- A4 latent RoPE / tables / query
    r = cases.rope_case()
    inv = s6_layer.latent_inv_freq(int(r['head_dim']), float(r['theta']))
    outs = dict(inv_freq=inv.numpy())
    pos = T_(r['positions'])
    for wd in (512, 256):
        table32 = s6_layer.latent_rope_table(int(r['max_pos']), inv, wd, torch.float32)
        table16 = s6_layer.latent_rope_table(int(r['max_pos']), inv, wd, torch.bfloat16)
        outs[f'table{wd}_rows'] = table32[pos].numpy()
        outs[f'table{wd}_bf16_rows'] = table16[pos].float().numpy()
        x = T_(r[f'x{wd}']).bfloat16()
        outs[f'rope{wd}_bf16'] = s6_ops.latent_rope(x, pos, table16, 'torch').float().numpy()
        outs[f'rope{wd}_f32'] = s6_ops.latent_rope(x.float(), pos, table32, 'torch').numpy()
        row = T_(r[f'row{wd}']).bfloat16()
        outs[f'rowrope{wd}_bf16'] = s6_ops.latent_rope(row[:, :wd], pos, table16, 'torch').float().numpy()
    save('rope', r, **outs)

    # ---- A9 writer: write_rows / committed_row in bf16 against LatentLayer.pack
    wc = cases.writer_case()
    hidden, rank, rank1 = wc['h'].shape[-1], int(wc['rank']), int(wc['rank1'])
    sl = LatentLayer(hidden, 16, 128, 4, rank, rank, rank1).to(torch.bfloat16)
    with torch.no_grad():
        for i in range(3):
            sl.cand_s[i].weight.copy_(T_(wc['E'][i]).bfloat16())
        sl.cand1.weight.copy_(T_(wc['E1']).bfloat16())
    pos = T_(wc['positions'])
    inv = s6_layer.latent_inv_freq(128, float(wc['theta']))
    tables = {wd: s6_layer.latent_rope_table(int(wc['max_pos']), inv, wd, torch.bfloat16) for wd in (rank, rank1)}

    class Ctx:
        positions = pos
        backends = s6_ops.TORCH_BACKENDS
    Ctx.tables = tables
    state, rows, regs = None, {}, []
    with torch.no_grad():
        hs = [T_(wc['h'][i]).bfloat16() for i in range(4)]
        for loop in range(4):
            state = s6_layer.write_rows(sl, loop, hs[loop], state)
            regs.append((state.reg if loop else state.first).float().numpy())
            row = s6_layer.committed_row(sl, loop, state, Ctx)
            if row is not None:
                rows[loop] = torch.cat(row, -1).float().numpy()
        emb = (pos[:, None].float() * inv[None]).repeat(1, 2)
        cos, sin = emb.cos().bfloat16(), emb.sin().bfloat16()
        packed = sl.pack(sl.write(hs)[-1], sl.write1(hs[0]), cos, sin).float().numpy()
    save('writer', wc, first=regs[0], reg1=regs[1], reg2=regs[2], reg3=regs[3], row_l1=rows[0], row_main=rows[3],
         packed=packed)

    # ---- contiguous-layout reader (HF engines)
    from hla.latent.fused_history import reference as contig_reference
    for name, kw in (('contig_512', dict(width=512)), ('contig_256', dict(seed=82, width=256, keys=37, batch=4))):
        cc = cases.contig_case(**kw)
        scale = 1 / math.sqrt(128)
        z, lse = contig_reference(T_(cc['q']), T_(cc['k']), T_(cc['v']), T_(cc['mask']).bool(), scale)
        save(name, cc, z=z.float().numpy(), lse=lse.float().numpy(), scale=np.float64(scale))

    # ---- per-head history read MLA-style (the LLA serving path)
    for name, kw in (('heads_lla', dict()), ('heads_gqa', dict(seed=102, kv_heads=4, rank=64, d_rope=32,
                                                              ctx=(40, 0, 16, 333)))):
        hc = cases.heads_case(**kw)
        r = int(hc['rank'])
        cache = T_(hc['cache'])
        ctx = T_(hc['ctx'])
        ws = s6_ops.S6Workspace(16, r, 64)          # unused by the torch backend
        o, lse = s6_ops.history_attention_kv(T_(hc['q']), cache, cache[..., :r], T_(hc['block_table']), ctx,
                                             1 / math.sqrt(128), 4, ws, None, None, 'torch', mla=True)
        save(name, hc, o=o.numpy(), lse=lse.numpy(), scale=np.float64(1 / math.sqrt(128)))

    # ---- rollout cache export (the reference exporter on a stand-in runner)
    import tempfile
    from types import SimpleNamespace as NS
    from hla.vllm_latent.cache_export import RolloutCacheExporter
    ec = cases.export_case()
    L, bs, length = ec['main'].shape[0], int(ec['block_size']), int(ec['length'])
    main = [T_(ec['main'][i]).bfloat16() for i in range(L)]
    l1 = [T_(ec['l1'][i]).bfloat16() for i in range(L)]
    names = [f'{i}.{kind}' for i in range(L) for kind in ('main', 'l1')]
    layers = [NS(self_attn=NS(attn_main=NS(layer_name=f'{i}.main', kv_cache=main[i]),
                              attn_l1=NS(layer_name=f'{i}.l1', kv_cache=l1[i]))) for i in range(L)]
    body = NS(latent_cfg=dict(num_layers=L), layers=layers)
    group_tables = [T_(ec['main_blocks'])[None], T_(ec['l1_blocks'])[None]]
    tables = [NS(num_blocks_per_row=[t.shape[1]], block_size=bs, get_cpu_tensor=(lambda t=t: t))
              for t in group_tables]
    batch = NS(req_id_to_index={'r': 0}, req_ids=['r'], num_computed_tokens_cpu=[0], block_table=tables)
    runner = NS(get_model=lambda: NS(model=body), speculative_config=None, input_batch=batch,
                kv_cache_config=NS(kv_cache_groups=[NS(layer_names=[n for n in names if n.endswith('main')]),
                                                    NS(layer_names=[n for n in names if n.endswith('l1')])]),
                requests={'r': NS(prompt_token_ids=list(range(length)))})
    runner._update_states = lambda schedule: None
    def execute(schedule):
        runner._update_states(schedule)
        runner.execute_model_state = NS(logits=torch.zeros(1, 4))
    runner.execute_model = execute
    with tempfile.TemporaryDirectory() as d:
        exporter = RolloutCacheExporter(runner)
        exporter.begin(Path(d) / 'v0', 0)
        runner.execute_model(NS(finished_req_ids=set(), num_scheduled_tokens={'r': length},
                                total_num_scheduled_tokens=length))
        ref = exporter.finish()['snapshots']['r']
        payload = torch.load(ref['path'], map_location='cpu', weights_only=True)
    assert payload['schema'] == 's6-rollout-cache-v1' and payload['length'] == length
    save('export', ec, rows=np.stack([r.float().numpy() for r in payload['rows']]))

    # ---- integer metadata
    mc = cases.meta_cases()
    meta = dict(
        token_requests=[[x.tolist() for x in s6_ops.token_requests(torch.tensor(qsl_, dtype=torch.int32), n)]
                        for qsl_, n in mc['token_requests']],
        history_lengths=[s6_ops.history_lengths(torch.tensor(a, dtype=torch.int32), torch.tensor(b, dtype=torch.int32)).tolist()
                         for a, b in mc['history_lengths']],
        num_kv_splits=[s6_ops.num_kv_splits(*c) for c in mc['num_kv_splits']],
    )
    (HERE / 'meta.json').write_text(json.dumps({'cases': {k: [list(map(lambda v: list(v) if isinstance(v, tuple) else v, c)) for c in mc[k]] for k in mc},
                                                'reference': meta}, indent=1))
    print('wrote meta.json')


if __name__ == '__main__':
    main()
