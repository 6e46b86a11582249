"""TEST INFRASTRUCTURE -- PyTorch-CPU restatement of mlip.cpp's PET model.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module; the product path never imports it.

mlip.cpp computes PET with ggml, which is not available here, so this module
restates the reference graph operation by operation in torch (fp32 by
default, fp64 for self-checks).  Forces and stress come from torch autograd
with respect to the padded edge vectors, exactly the leaf the reference
differentiates.  Each step cites the reference code it follows:

  batch preparation ........ src/models/pet/pet_batch.cpp:54-666
    neighbour lists          oracle/nl.py (bit-exact with the reference NL)
    NEF padding, slot order  pet_batch.cpp:260-394 (stable sort by centre)
    reverse-edge map         pet_batch.cpp:399-565 ((i,j,S) -> (j,i,-S))
    attention mask           pet_batch.cpp:570-666 (fp16 log(cutoff), -inf pad)
    smooth cutoff (mask)     pet_batch.cpp:37-47
  in-graph r, f_c .......... src/models/pet/pet.cpp:203-256
  initial embeddings ....... pet.cpp:789-832
  GNN layer ................ pet.cpp:834-914
    edge embedding           pet_layers.cpp:151-217
    token compression        pet_layers.cpp:685-796
    attention                pet_layers.cpp:318-492 (QKV split [q;k;v], heads)
    transformer block        pet_layers.cpp:242-298 (post-LN)
    layer norm               pet_layers.cpp:85-145 (var * (1 + eps))
  reversed message avg ..... pet_layers.cpp:608-679, pet.cpp:726-729
  readout .................. pet_layers.cpp:920-1015
  energy assembly .......... pet.cpp:533-568 (double sum + composition)
  forces ................... pet.cpp:916-999
  stress ................... pet.cpp:1001-1098

Parity with ggml itself is unpinned (no ggml here); the restatement is
pinned instead by finite-difference forces and stress, momentum
conservation, batch == single and invariance tests in tests/.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import nl as _nl


# --------------------------------------------------------------------------
# Batch preparation (pet_batch.cpp)
# --------------------------------------------------------------------------
def smooth_cutoff_f32(r: np.ndarray, rc: float, delta: float) -> np.ndarray:
    """pet_batch.cpp:37-47 in float32."""
    r = np.asarray(r, np.float32)
    rc32, d32 = np.float32(rc), np.float32(delta)
    x = (r - rc32 + d32) / d32
    mid = np.float32(0.5) + np.float32(0.5) * np.cos(np.float32(math.pi) * x).astype(np.float32)
    out = np.where(r >= rc32, np.float32(0), np.where(r <= rc32 - d32, np.float32(1), mid))
    return out.astype(np.float32)


@dataclass
class Batch:
    n_atoms: int
    n_systems: int
    max_nb: int
    species: np.ndarray          # [N] species index
    system: np.ndarray           # [N] system index
    vec: np.ndarray              # [N, M, 3] float32 NEF edge vectors (0 for pad)
    nbr_species: np.ndarray      # [N, M] (pad -> 0)
    pad: np.ndarray              # [N, M] float32 1 = real
    nbr: np.ndarray              # [N, M] neighbour atom (pad -> 0)
    rev_flat: np.ndarray         # [N, M] j*M + k' (no reverse -> 0)
    rev_mask: np.ndarray         # [N, M] float32
    key_mask: np.ndarray         # [N, 1+M] float32 values of the fp16 mask
    atoms_per_system: list
    numbers: np.ndarray          # [N] atomic numbers


def prepare_batch(systems, cutoff: float, cutoff_width: float, species_to_index: dict) -> Batch:
    """prepare_batch (pet_batch.cpp:670-761) for a list of Structure-like
    objects (positions, numbers, cell, pbc)."""
    nls, offs, n_tot = [], [], 0
    for s in systems:
        nls.append(_nl.build_oracle(s.positions, s.cell, s.pbc, cutoff))
        offs.append(n_tot)
        n_tot += len(s.positions)
    N = n_tot
    centers = np.concatenate([l["centers"] + o for l, o in zip(nls, offs)]) if N else np.zeros(0, np.int32)
    nbrs = np.concatenate([l["neighbors"] + o for l, o in zip(nls, offs)])
    shifts = np.concatenate([l["cell_shifts"] for l in nls])
    vecs = np.concatenate([l["edge_vectors"] for l in nls])
    dists = np.concatenate([l["distances"] for l in nls])
    numbers = np.concatenate([np.asarray(s.numbers, np.int32) for s in systems])
    system = np.concatenate([np.full(len(s.positions), k, np.int32) for k, s in enumerate(systems)])
    try:
        species = np.array([species_to_index[int(z)] for z in numbers], np.int32)
    except KeyError as e:
        raise ValueError(f"Unknown atomic number {e.args[0]} not found in species_to_index mapping")
    E = len(centers)
    cnt = np.bincount(centers, minlength=N) if E else np.zeros(N, np.int64)
    M = int(max(1, cnt.max() if N else 1))
    order = np.argsort(centers, kind="stable")           # pet_batch.cpp:283-289
    eoff = np.concatenate([[0], np.cumsum(cnt)])
    slot_of = np.empty(E, np.int64)
    slot_of[order] = np.arange(E) - eoff[centers[order]]
    flat = centers.astype(np.int64) * M + slot_of         # NEF position of each edge
    vec = np.zeros((N * M, 3), np.float32); vec[flat] = vecs
    pad = np.zeros(N * M, np.float32); pad[flat] = 1
    nbr = np.zeros(N * M, np.int32); nbr[flat] = nbrs
    nsp = np.zeros(N * M, np.int32); nsp[flat] = species[nbrs]
    dnl = np.zeros(N * M, np.float32); dnl[flat] = dists
    # reverse map: key (i, j, S) -> edge; reverse of e is key (j, i, -S)
    rev_flat = np.zeros(N * M, np.int64)
    rev_mask = np.zeros(N * M, np.float32)
    if E:
        def key(i, j, s):
            b = 1 << 10
            sh = (s + b // 2).astype(np.int64)
            return (((i.astype(np.int64) * N + j) * b + sh[:, 0]) * b + sh[:, 1]) * b + sh[:, 2]
        k_fwd = key(centers, nbrs, shifts)
        k_rev = key(nbrs, centers, -shifts)
        srt = np.argsort(k_fwd, kind="stable")
        pos = np.searchsorted(k_fwd[srt], k_rev)
        pos = np.minimum(pos, E - 1)
        hit = k_fwd[srt][pos] == k_rev
        r_e = srt[pos]
        rev_flat[flat[hit]] = flat[r_e[hit]]
        rev_mask[flat[hit]] = 1
    # attention key mask (pet_batch.cpp:603-653): key 0 = node, keys 1..M edges
    fc = smooth_cutoff_f32(dnl, cutoff, cutoff_width)
    val = np.where((pad > 0.5) & (fc > 0), fc, np.float32(0))
    with np.errstate(divide="ignore"):
        logv = np.where(val > 0, np.log(np.maximum(val, np.float32(1e-45))).astype(np.float32), -np.inf)
    key_mask = np.empty((N, 1 + M), np.float32)
    key_mask[:, 0] = 0.0
    key_mask[:, 1:] = logv.reshape(N, M).astype(np.float16).astype(np.float32)
    return Batch(N, len(systems), M, species, system, vec.reshape(N, M, 3), nsp.reshape(N, M),
                 pad.reshape(N, M), nbr.reshape(N, M), rev_flat.reshape(N, M),
                 rev_mask.reshape(N, M), key_mask, [len(s.positions) for s in systems], numbers)


# --------------------------------------------------------------------------
# Model
# --------------------------------------------------------------------------
class PETOracle:
    """CPU restatement of PETModel (src/models/pet/pet.cpp)."""

    def __init__(self, hypers, tensors: dict, dtype=torch.float32):
        self.h = hypers
        self.dtype = dtype
        self.W = {k: torch.as_tensor(np.asarray(v)).to(dtype) for k, v in tensors.items()
                  if v.dtype != np.int32}
        z = np.asarray(tensors["composition.atomic_numbers"], np.int32)
        e = np.asarray(tensors["composition.energies"], np.float32)
        self.species_to_index = {int(a): i for i, a in enumerate(z)}
        self.composition = {int(a): float(b) for a, b in zip(z, e)}

    # pet_layers.cpp:85-145 -- LN with var * (1 + eps)
    @staticmethod
    def _ln(x, w, b, eps=1e-5):
        mu = x.mean(-1, keepdim=True)
        xc = x - mu
        var = (xc * xc).mean(-1, keepdim=True)
        return xc / torch.sqrt(var * (1.0 + eps)) * w + b

    def _lin(self, x, name):
        return x @ self.W[name + ".weight"].T + self.W[name + ".bias"]

    # pet_types.h:247-254 (has_property): a property is present when its
    # layer-0 node head is; pet_types.h:101 (is_loaded) per layer
    NC_PROPS = {"nc_forces": ("nc_f", 3), "nc_stress": ("nc_s", 9)}

    def has_property(self, prop: str, layer: int = 0) -> bool:
        return f"model.node_heads.{prop}.{layer}.0.weight" in self.W

    def atomic_energies(self, b: Batch, vec: torch.Tensor, nc: bool = False):
        """Per-atom energies; with nc also the per-atom non-conservative
        outputs {prop: [N, od]} of the properties the model has."""
        h, W = self.h, self.W
        N, M = b.n_atoms, b.max_nb
        d, nh = h.d_pet, h.num_heads
        hd = d // nh
        sp = torch.as_tensor(b.species, dtype=torch.long)
        nsp = torch.as_tensor(b.nbr_species, dtype=torch.long)
        pad = torch.as_tensor(b.pad, dtype=self.dtype)
        # pet.cpp:208-256: r and f_c computed in-graph from the leaf
        r = torch.sqrt((vec * vec).sum(-1))
        inv_delta = 1.0 / h.cutoff_width
        off = (h.cutoff_width - h.cutoff) * inv_delta
        xc = torch.clamp(r * inv_delta + off, 0.0, 1.0)
        fc = 0.5 * torch.cos(math.pi * xc) + 0.5
        mask = torch.as_tensor(b.key_mask, dtype=self.dtype)[:, None, None, :]   # [N,1,1,S]
        m0 = W["model.embedding.weight"][nsp]                                    # [N,M,d]
        msg = m0
        energies = torch.zeros(N, dtype=self.dtype)
        props = [p for p in self.NC_PROPS if nc and self.has_property(p)]
        nc_out = {p: torch.zeros(N, self.NC_PROPS[p][1], dtype=self.dtype) for p in props}
        edge0 = None
        for l in range(2):
            p = f"model.gnn.{l}."
            we = W[p + "edge_embedder.weight"]
            emb = vec @ we[:, :3].T + r[..., None] * we[:, 3] + W[p + "edge_embedder.bias"]
            parts = [emb] if l == 0 else [emb, W[p + "neighbor_embedder.weight"][nsp]]
            cat = torch.cat(parts + [msg], -1)
            tok = self._lin(torch.nn.functional.silu(self._lin(cat, p + "compress.0")), p + "compress.2")
            node = W[p + "node_embedder.weight"][sp]
            x = torch.cat([node[:, None, :], tok], 1)                            # [N,S,d]
            S = M + 1
            for t in range(2):
                q_ = p + f"tl.{t}."
                qkv = self._lin(x, q_ + "attn.in").reshape(N, S, 3, nh, hd)
                q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))      # [N,nh,S,hd]
                s = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(hd)) + mask
                a = torch.softmax(s, -1) @ v                                      # [N,nh,S,hd]
                a = a.transpose(1, 2).reshape(N, S, d)
                x = self._ln(x + self._lin(a, q_ + "attn.out"), W[q_ + "norm_a.weight"], W[q_ + "norm_a.bias"])
                hmid = torch.nn.functional.silu(self._lin(x, q_ + "mlp.0"))
                x = self._ln(x + self._lin(hmid, q_ + "mlp.3"), W[q_ + "norm_m.weight"], W[q_ + "norm_m.bias"])
            node_f, edge_f = x[:, 0], x[:, 1:]
            if l == 0:
                edge0 = edge_f
                rev = torch.as_tensor(b.rev_flat, dtype=torch.long).reshape(-1)
                rm = torch.as_tensor(b.rev_mask, dtype=self.dtype)[..., None]
                msg = 0.5 * (m0 + rm * edge0.reshape(N * M, d)[rev].reshape(N, M, d))
            energies = energies + self._head(node_f, "node", l) + \
                (self._head(edge_f, "edge", l) * fc * pad).sum(-1)
            # build_property_output (pet_layers.cpp:845-915): node head plus
            # the cutoff- and padding-weighted edge head summed over neighbours
            for p in props:
                if self.has_property(p, l):
                    nc_out[p] = nc_out[p] + self._prop_head(node_f, "node", p, l) + \
                        (self._prop_head(edge_f, "edge", p, l) * (fc * pad)[..., None]).sum(1)
        return (energies, nc_out) if nc else energies

    def _prop_head(self, x, kind, prop, l):
        """apply_mlp_head (pet_layers.cpp:811-837) of a property head."""
        hp = f"model.{kind}_heads.{prop}.{l}."
        y = torch.nn.functional.silu(self._lin(x, hp + "0"))
        y = torch.nn.functional.silu(self._lin(y, hp + "2"))
        return self._lin(y, f"model.{kind}_last_layers.{prop}.{l}.{self.NC_PROPS[prop][0]}")

    def _head(self, x, kind, l):
        hp = f"model.{kind}_heads.energy.{l}."
        y = torch.nn.functional.silu(self._lin(x, hp + "0"))
        y = torch.nn.functional.silu(self._lin(y, hp + "2"))
        return self._lin(y, f"model.{kind}_last_layers.energy.{l}.energy___0")[..., 0]

    # ----------------------------------------------------------------------
    def predict(self, systems, compute_forces=True, key_mask=None, compute_nc=False):
        """predict_batch (pet.cpp:125-694): list of dicts with energy
        (python float, f32-rounded like ModelResult), forces [n,3] and stress
        [6] (Voigt xx,yy,zz,yz,xz,xy) when available.

        compute_nc runs the non-conservative heads the model has: their
        per-atom forces are added to the forces (zero without gradients),
        their per-atom stress tensors summed per system into Voigt form,
        added to the stress and the sum divided by the volume for periodic
        systems (pet.cpp:576-686).

        The reference's attention mask is an input built from the neighbour
        list distances, so its forces omit the mask's position dependence.
        `key_mask` (a Batch.key_mask) lets finite-difference checks hold the
        mask fixed the same way."""
        if not isinstance(systems, (list, tuple)):
            systems = [systems]
        h = self.h
        b = prepare_batch(systems, h.cutoff, h.cutoff_width, self.species_to_index)
        if key_mask is not None:
            b.key_mask = key_mask
        vec = torch.as_tensor(b.vec, dtype=self.dtype).clone().requires_grad_(compute_forces)
        with torch.set_grad_enabled(compute_forces):
            e_at = self.atomic_energies(b, vec, nc=compute_nc)
            nc_out = {}
            if compute_nc:
                e_at, nc_out = e_at
            if compute_forces:
                (g,) = torch.autograd.grad(e_at.sum(), vec)
        e_np = e_at.detach().to(torch.float32).numpy()
        results = []
        off = 0
        for k, s in enumerate(systems):
            n = len(s.positions)
            tot = float(np.sum(e_np[off:off + n].astype(np.float64)))
            for z in s.numbers:
                tot += self.composition.get(int(z), 0.0)
            res = {"energy": float(np.float32(tot)), "energy_f64": tot}
            results.append(res)
            off += n
        if compute_forces:
            g = g.detach().numpy()
            valid = b.pad > 0.5
            F = np.zeros((b.n_atoms, 3), np.float64)
            ci = np.repeat(np.arange(b.n_atoms), b.max_nb).reshape(b.n_atoms, b.max_nb)
            np.add.at(F, ci[valid], g[valid])
            np.add.at(F, b.nbr[valid], -g[valid])
            vir = np.zeros((b.n_systems, 6))
            e = b.vec[valid].astype(np.float64)
            gv = g[valid].astype(np.float64)
            sysid = b.system[ci[valid]]
            comps = [e[:, 0] * gv[:, 0], e[:, 1] * gv[:, 1], e[:, 2] * gv[:, 2],
                     0.5 * (e[:, 1] * gv[:, 2] + e[:, 2] * gv[:, 1]),
                     0.5 * (e[:, 0] * gv[:, 2] + e[:, 2] * gv[:, 0]),
                     0.5 * (e[:, 0] * gv[:, 1] + e[:, 1] * gv[:, 0])]
            for c in range(6):
                np.add.at(vir[:, c], sysid, comps[c])
            off = 0
            for k, s in enumerate(systems):
                n = len(s.positions)
                results[k]["forces"] = F[off:off + n].astype(np.float32)
                off += n
                if s.cell is not None and (s.pbc is None or any(s.pbc)):
                    m = np.asarray(s.cell, np.float32)
                    vol = abs(float(np.float32(m[0, 0] * (m[1, 1] * m[2, 2] - m[1, 2] * m[2, 1]) -
                                               m[0, 1] * (m[1, 0] * m[2, 2] - m[1, 2] * m[2, 0]) +
                                               m[0, 2] * (m[1, 0] * m[2, 1] - m[1, 1] * m[2, 0]))))
                    if vol > 1e-10:
                        results[k]["stress"] = (vir[k] / vol).astype(np.float32)
        if "nc_forces" in nc_out:
            ncf = nc_out["nc_forces"].detach().numpy()
            off = 0
            for k, s in enumerate(systems):
                n = len(s.positions)
                base = results[k].get("forces", np.zeros((n, 3), np.float32))
                results[k]["forces"] = (base + ncf[off:off + n]).astype(np.float32)
                off += n
        if "nc_stress" in nc_out:
            t = nc_out["nc_stress"].detach().numpy().astype(np.float64)
            voigt = np.stack([t[:, 0], t[:, 4], t[:, 8], 0.5 * (t[:, 5] + t[:, 7]),
                              0.5 * (t[:, 2] + t[:, 6]), 0.5 * (t[:, 1] + t[:, 3])], 1)
            off = 0
            for k, s in enumerate(systems):
                n = len(s.positions)
                st = results[k].get("stress", np.zeros(6, np.float32)).astype(np.float64)
                st = st + voigt[off:off + n].sum(0)
                off += n
                if s.cell is not None and (s.pbc is None or any(s.pbc)):
                    m = np.asarray(s.cell, np.float32)
                    vol = abs(float(np.float32(m[0, 0] * (m[1, 1] * m[2, 2] - m[1, 2] * m[2, 1]) -
                                               m[0, 1] * (m[1, 0] * m[2, 2] - m[1, 2] * m[2, 0]) +
                                               m[0, 2] * (m[1, 0] * m[2, 1] - m[1, 1] * m[2, 0]))))
                    if vol > 1e-10:
                        results[k]["stress"] = (st / vol).astype(np.float32)
        return results


def load_oracle(gguf_path: str, dtype=torch.float32) -> PETOracle:
    import importlib
    import sys
    wl = sys.modules.get("mlipcpp_b200.workloads") or importlib.import_module("mlipcpp_b200.workloads")
    h, t = wl.read_pet_gguf(gguf_path)
    return PETOracle(h, t, dtype)
