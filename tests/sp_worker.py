"""Worker of tests/test_parallel_gpu.py (run under torchrun): the Ulysses engine on WORLD_SIZE GPUs against the
single-GPU engine on the same seeded inputs and weights, over three forwards (dynamic, then delayed scales).  With
SP_MASK=1 both engines run attention under the same seeded block-sparse mask; SP_QKV_PARTS=k splits the qkv GEMM and
its exchange into k row parts and SP_PART_SENDER=copy|push picks how the parts are sent (the engine's defaults
otherwise)."""
import os, sys
from datetime import timedelta
root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(root, "minimax-h3-tensorfold-rtx_b200")); sys.path.insert(0, root)
import torch, torch.distributed as dist
rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
from tfvideo import attention as A, minimax_h3 as M, native as N
cfg = M.Config(layers=2, dim=512, heads=8, head_dim=128, ffn=1024, act="gelu", t_dim=8)
S = 1024
g = torch.Generator().manual_seed(5)
x = torch.randn(S, cfg.dim, generator=g).to(torch.bfloat16).cuda()
t_emb = torch.randn(2, cfg.t_dim, generator=g).cuda()
segs = [(0, 100, 0), (100, S, 3)]
rot = 128
ang = torch.randn(S, rot // 2, generator=g)
rope = torch.stack([torch.stack([ang.cos(), -ang.sin()], -1), torch.stack([ang.sin(), ang.cos()], -1)], -2)
rope = rope.reshape(1, S, 1, rot // 2, 2, 2).cuda()
eng = M.MiniMaxH3Engine.synthetic(cfg, seed=1, device="cuda", group=dist.group.WORLD)
mask = A.TileMask.block_sparse(S, keep=0.5, text_tokens=128, seed=3) if os.environ.get("SP_MASK") == "1" else None
eng.attn_mask = mask
if os.environ.get("SP_QKV_PARTS"):
    eng.qkv_parts = int(os.environ["SP_QKV_PARTS"])
if os.environ.get("SP_PART_SENDER"):
    eng.part_sender = os.environ["SP_PART_SENDER"]
n = S // world
outs = []
for f in range(3):
    xs = x[rank * n:(rank + 1) * n].clone()
    outs.append(eng.forward(xs, t_emb, segs, rope).clone())
gath = [torch.empty_like(outs[-1]) for _ in range(world)]
dist.all_gather(gath, outs[-1])
full_sp = torch.cat(gath)
if rank == 0:
    ref = M.MiniMaxH3Engine.from_weights(M.synthetic_weights(cfg, 1, "cuda"), cfg, device="cuda")
    ref.sp = None
    ref.attn_mask = mask
    for f in range(3):
        r = ref.forward(x.clone(), t_emb, segs, rope)
    torch.cuda.synchronize()
    eq = torch.equal(full_sp, r)
    cos = torch.nn.functional.cosine_similarity(full_sp.float().flatten(), r.float().flatten(), dim=0).item()
    print(f"RESULT world={world} mask={mask is not None} bitwise={eq} cosine={cos:.8f} status={N.device_status()}",
          flush=True)
dist.barrier()
dist.destroy_process_group()
