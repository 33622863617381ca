"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no dataset for this path; these generators stand in
with the shapes and value distributions of the configurations it is measured
on (logits [B, C] fp32, labels int64 uniform in [0, C)).  All draws come from
a CPU torch.Generator in a fixed order, so the same (config, rows) gives the
same tensors on every host where torch runs the same CPU kernels: its float32
normal kernel gives other values where it runs its scalar code than where it
runs the AVX2/AVX-512 one (the parity tests compare with the reference's
golden outputs only when the input fingerprint matches, and always with the
oracle on the same inputs).

  cfg0  256 x 100      N(0,1)                                     seed 0
  cfg1  4096 x 1000    N(0,1), +4.0 at the label                  seed 1
  cfg2  4096 x 32000   Student-t (df 3, scale 2)                  seed 2
  cfg3  65536 x 128    8 levels {-3.5..3.5}, 1% set to +-0.0      seed 3
  cfg4  8192 x 128256  N(0,1), +8.0 at one non-label class        seed 4
                       (generated per 1024-row block, seed 4*1000003+block,
                       so any row block can be generated alone)
"""
import torch

CONFIGS = {
    "cfg0": (256, 100),
    "cfg1": (4096, 1000),
    "cfg2": (4096, 32000),
    "cfg3": (65536, 128),
    "cfg4": (8192, 128256),
}
CFG4_BLOCK = 1024


def _gen(seed):
    return torch.Generator().manual_seed(int(seed))


def _cfg0(B, C, g):
    z = torch.randn(B, C, generator=g)
    y = torch.randint(0, C, (B,), generator=g)
    return z, y


def _cfg1(B, C, g):
    z = torch.randn(B, C, generator=g)
    y = torch.randint(0, C, (B,), generator=g)
    z[torch.arange(B), y] += 4.0
    return z, y


def _cfg2(B, C, g):
    # Student-t(3) * 2 built from one generator (torch.distributions.StudentT
    # takes no generator): n / sqrt(chi2_3 / 3).
    n = torch.randn(B, C, generator=g)
    c = torch.zeros(B, C)
    for _ in range(3):
        c.add_(torch.randn(B, C, generator=g).square_())
    z = n.mul_(2.0).div_(c.div_(3.0).sqrt_())
    y = torch.randint(0, C, (B,), generator=g)
    return z, y


def _cfg3(B, C, g):
    levels = torch.arange(-3.5, 4.0, 1.0)
    z = levels[torch.randint(0, 8, (B, C), generator=g)]
    m = torch.rand(B, C, generator=g) < 0.01
    s = torch.rand(B, C, generator=g) < 0.5
    zeros = torch.where(s, torch.tensor(0.0), torch.tensor(-0.0))
    z = torch.where(m, zeros, z)
    y = torch.randint(0, C, (B,), generator=g)
    return z.contiguous(), y


def _cfg4_block(block, rows, C):
    g = _gen(4 * 1000003 + block)
    z = torch.randn(rows, C, generator=g)
    y = torch.randint(0, C, (rows,), generator=g)
    b = (y + torch.randint(1, C, (rows,), generator=g)) % C
    z[torch.arange(rows), b] += 8.0
    return z, y


def shape_of(name):
    """(B, C) of a configuration name: cfg0..cfg4 or 'gaussBxC'."""
    return parse_gaussian(name) or CONFIGS[name]


def make_gaussian(B, C, sigma=1.0, seed=0):
    """N(0, sigma^2) logits [B, C] and uniform labels: the reference's CUDA
    benchmark workload (benchmarks/cuda_benchmarks/CE_FW_perf.py, B = 32)."""
    g = _gen(seed)
    z = torch.randn(B, C, generator=g) * float(sigma)
    y = torch.randint(0, C, (B,), generator=g)
    return z, y


def parse_gaussian(name):
    """'gaussBxC' -> (B, C), else None (bench configurations of that form)."""
    if not name.startswith("gauss"):
        return None
    B, C = name[5:].split("x")
    return int(B), int(C)


def make_rank(name, rank):
    """The batch of one rank under weak scaling: rank 0 gets the configuration
    itself, rank r > 0 the same recipe with its own rows (cfg4: row blocks
    r*B.. of the block-seeded stream; others: seed + 7919 r)."""
    shape = parse_gaussian(name)
    if shape:
        return make_gaussian(*shape, seed=rank)
    if rank == 0:
        return make(name)
    B, C = CONFIGS[name]
    if name == "cfg4":
        return make_cfg4_rows(rank * B, (rank + 1) * B, C)
    fn = {"cfg0": _cfg0, "cfg1": _cfg1, "cfg2": _cfg2, "cfg3": _cfg3}[name]
    return fn(B, C, _gen(int(name[3:]) + 7919 * rank))


def make(name, rows=None, cols=None):
    """(logits fp32 [B, C], labels int64 [B]) on the CPU.

    `rows`/`cols` shrink the configuration (same recipe and seed, fewer rows or
    classes); for cfg4, `rows` selects the first row blocks and a partial last
    block (each block from its own seed)."""
    shape = parse_gaussian(name)
    if shape:
        return make_gaussian(shape[0] if rows is None else int(rows), shape[1] if cols is None else int(cols))
    B, C = CONFIGS[name]
    B = B if rows is None else int(rows)
    C = C if cols is None else int(cols)
    seed = int(name[3:])
    if name == "cfg4":
        return make_cfg4_rows(0, B, C)
    return {"cfg0": _cfg0, "cfg1": _cfg1, "cfg2": _cfg2, "cfg3": _cfg3}[name](B, C, _gen(seed))


def make_cfg4_rows(start, stop, C=None):
    """Rows [start, stop) of cfg4 (start must be a multiple of 1024)."""
    C = CONFIGS["cfg4"][1] if C is None else int(C)
    assert start % CFG4_BLOCK == 0, "cfg4 shards start on 1024-row blocks"
    zs, ys = [], []
    r = start
    while r < stop:
        blk = r // CFG4_BLOCK
        n = min(CFG4_BLOCK, stop - r)
        z, y = _cfg4_block(blk, CFG4_BLOCK, C) if n == CFG4_BLOCK else _cfg4_block(blk, n, C)
        zs.append(z)
        ys.append(y)
        r += n
    return torch.cat(zs), torch.cat(ys)
