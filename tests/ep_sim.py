"""Host restatement of the expert-parallel exchange (rusty_engine_b200/csrc/ep.cu) for the CPU
tests: the same placement (the caller's expert -> rank table, or round-robin e % G; local ids
in ascending global order), the same plan (each
token sent once to every rank holding one of its picks, in token order), the same row contents (the token and its picks as seen by the destination: local
expert id or the empty id = the destination's expert count, and the weight), the same per-row partial sums and the same
combine order (ascending rank), with torch.distributed all-to-all standing in for NCCL.
Expert math is the oracle's exact f32 path.  Test infrastructure only."""
import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle as O


def placement_tables(E: int, G: int, placement=None):
    """rank_of[e], local_of[e] and the experts of each rank (ascending) for a placement table
    (None: round-robin, expert e on rank e % G)."""
    rank_of = np.array([e % G for e in range(E)] if placement is None else placement, dtype=np.int64)
    held = [[e for e in range(E) if rank_of[e] == d] for d in range(G)]
    local_of = np.zeros(E, dtype=np.int64)
    for d in range(G):
        for j, e in enumerate(held[d]):
            local_of[e] = j
    return rank_of, local_of, held


def plan(ids: np.ndarray, G: int, self_all: int = -1, rank_of=None):
    """pos[t, d] = row of token t in d's block (-1 when not sent), counts[d]; expert e lives
    on rank rank_of[e] (e % G when not given); every token also goes to rank `self_all` when
    that is >= 0 (the home rank, which runs the shared expert)."""
    T = ids.shape[0]
    flags = np.zeros((T, G), dtype=bool)
    for t in range(T):
        for e in ids[t]:
            flags[t, int(e) % G if rank_of is None else int(rank_of[int(e)])] = True
        if self_all >= 0:
            flags[t, self_all] = True
    pos = np.full((T, G), -1, dtype=np.int64)
    counts = np.zeros(G, dtype=np.int64)
    for d in range(G):
        for t in range(T):
            if flags[t, d]:
                pos[t, d] = counts[d]
                counts[d] += 1
    return pos, counts


def a2a(rows: np.ndarray, send_counts, recv_counts, width: int) -> np.ndarray:
    out = torch.empty((int(sum(recv_counts)), width), dtype=torch.float64)
    dist.all_to_all_single(out, torch.from_numpy(np.ascontiguousarray(rows, dtype=np.float64)).reshape(-1, width),
                           output_split_sizes=[int(c) for c in recv_counts],
                           input_split_sizes=[int(c) for c in send_counts])
    return out.numpy()


def ep_forward(x: np.ndarray, layer, experts_f32, rank: int, G: int, shared_f32=None, placement=None) -> np.ndarray:
    """This rank's tokens x [T, H] -> layer outputs [T, H]; experts_f32[e] = (gate, up, down);
    shared_f32 = the shared expert's (gate, up, down), replicated on every rank; placement[e] =
    the rank holding expert e (None: round-robin)."""
    T, H = x.shape
    E, k, I = layer.E, layer.k, layer.I
    rank_of, local_of, held = placement_tables(E, G, placement)
    El = len(held[rank])
    logits = O.router_logits(x, layer.router_w, E)
    ids, w = O.route_batch(logits, layer.gate, k)
    pos, send_counts = plan(ids, G, rank if shared_f32 is not None else -1, rank_of)
    recv_counts = torch.empty(G, dtype=torch.int64)
    dist.all_to_all_single(recv_counts, torch.from_numpy(send_counts))
    recv_counts = recv_counts.numpy()
    # rows: [x (H) | local ids (k) | weights (k)], grouped by destination, token order inside
    width = H + 2 * k
    soff = np.concatenate([[0], np.cumsum(send_counts)])
    rows = np.zeros((int(soff[-1]), width))
    for t in range(T):
        for d in range(G):
            if pos[t, d] < 0:
                continue
            r = soff[d] + pos[t, d]
            rows[r, :H] = x[t]
            for j in range(k):
                mine = rank_of[int(ids[t, j])] == d
                rows[r, H + j] = local_of[int(ids[t, j])] if mine else len(held[d])
                rows[r, H + k + j] = w[t, j] if mine else 0.0
    got = a2a(rows, send_counts, recv_counts, width)
    # local experts: per received row, the weighted sum of its picks held here; the rows this
    # rank sent itself also take the shared expert at weight 1
    roff = np.concatenate([[0], np.cumsum(recv_counts)])
    part = np.zeros((got.shape[0], H))
    for r in range(got.shape[0]):
        xr = got[r, :H].astype(np.float32)
        if shared_f32 is not None and roff[rank] <= r < roff[rank + 1]:
            part[r] += O.expert_ffn(xr, *shared_f32, H, I).astype(np.float64)
        for j in range(k):
            le = int(got[r, H + j])
            if le >= El:
                continue
            g, u, dn = experts_f32[held[rank][le]]
            part[r] += got[r, H + k + j] * O.expert_ffn(xr, g, u, dn, H, I).astype(np.float64)
    back = a2a(part, recv_counts, send_counts, H)
    out = np.zeros((T, H))
    for t in range(T):
        for d in range(G):  # ascending rank
            if pos[t, d] >= 0:
                out[t] += back[soff[d] + pos[t, d]]
    return out.astype(np.float32)
