"""Full-size synthetic MoE layers generated on the device.

The weights follow the reference's synthetic-model recipe (N(0, 0.02) floats
quantised by BlockQuantizer; src/QuantRunner.Cli/Program.cs:357-362): every
matrix is drawn by qrm_synth_gaussian from its own seed and quantised on the
device by qrm_synth_quantize, whose bytes equal the CPU quantiser's
(tests/test_gpu_synth.py).  So any expert can be regenerated from its seed,
on any rank, without being held: the oracle gets host bytes of exactly the
experts a batch selects.

`pool` (optional) makes expert e reuse the matrices of expert e % pool, which
keeps host-side copies small for the parity tests; routing still ranges over
all n_experts (the router rows are distinct).
"""
import numpy as np

from tests.moe_case import CONFIGS, MoeCase, storage_fmt

SEED_BASE = 0x51520000


class SynthLayer:
    def __init__(self, name, seed=None, pool=None, weight_sigma=0.02, router_sigma=0.02, norm_random=False,
                 **over):
        cfg = dict(CONFIGS[name])
        cfg.update(over)
        self.name = name
        self.cfg = cfg
        self.seed = seed if seed is not None else SEED_BASE + int(name[1:]) * 0x100
        self.pool = pool
        self.weight_sigma = weight_sigma
        self.router_sigma = router_sigma
        self.norm_random = norm_random
        self.qfmt = tuple(cfg["fmt"])                          # quantiser ids (108 = TriLegacy)
        self.fmt = tuple(storage_fmt(f) for f in self.qfmt)    # storage format ids
        self.shared = cfg["n_shared"] > 0 and bool(cfg["moe_sigmoid"])
        self.qfmt_sh = tuple(cfg.get("shared_fmt", self.qfmt))
        self.fmt_sh = tuple(storage_fmt(f) for f in self.qfmt_sh) if self.shared else (0, 0, 0)
        self._host = {}
        self._small = None

    # ---------------------------------------------------------------- seeds
    def matrix_seed(self, expert, which):
        E = self.cfg["n_experts"]
        if expert < 0:
            return self.seed * 4096 + E * 3 + which
        p = expert % self.pool if self.pool else expert
        return self.seed * 4096 + p * 3 + which

    def shape(self, which):
        d, f = self.cfg["d_model"], self.cfg["expert_ffn"]
        return (d, f) if which == 2 else (f, d)

    # ---------------------------------------------------------------- device
    def _bufs(self, torch, Q, dev):
        d, f = self.cfg["d_model"], self.cfg["expert_ffn"]
        n = d * f
        if getattr(self, "_tmp", None) is None or self._tmp.device.index != dev:
            self._tmp = torch.empty(n, dtype=torch.float32, device=f"cuda:{dev}")
            self._qbuf = torch.empty(Q.tensor_bytes(n, 4), dtype=torch.uint8, device=f"cuda:{dev}")
        return n

    def synth_matrix(self, torch, Q, dev, expert, which):
        """Quantised bytes of one matrix on the device (a view of a scratch
        buffer, valid until the next call) and their count."""
        n = self._bufs(torch, Q, dev)
        qf = (self.qfmt_sh if expert < 0 else self.qfmt)[which]
        Q.synth_gaussian(self._tmp.data_ptr(), n, self.matrix_seed(expert, which), self.weight_sigma)
        Q.synth_quantize(qf, self._tmp.data_ptr(), n, self._qbuf.data_ptr())
        return self._qbuf, Q.tensor_bytes(n, qf)

    def host_matrix(self, torch, Q, dev, expert, which):
        key = (expert if expert < 0 or not self.pool else expert % self.pool, which)
        if key not in self._host:
            q, nb = self.synth_matrix(torch, Q, dev, expert, which)
            self._host[key] = q[:nb].cpu().numpy().copy()
        return self._host[key]

    def small_tensors(self, torch, Q, dev):
        """Router [E x d], bias [E] or None, offset [E] or None, norm [d] (host)."""
        if self._small is None:
            c = self.cfg
            E, d = c["n_experts"], c["d_model"]
            buf = torch.empty(E * d, dtype=torch.float32, device=f"cuda:{dev}")
            Q.synth_gaussian(buf.data_ptr(), E * d, self.seed + 1, self.router_sigma)
            router = buf.cpu().numpy().reshape(E, d).copy()
            bias = offset = None
            if c.get("bias_sigma"):
                Q.synth_gaussian(buf.data_ptr(), E, self.seed + 2, c["bias_sigma"])
                bias = buf[:E].cpu().numpy().copy()
            if c.get("offset_sigma"):
                Q.synth_gaussian(buf.data_ptr(), E, self.seed + 3, c["offset_sigma"])
                offset = buf[:E].cpu().numpy().copy()
            norm = np.ones(d, np.float32)
            if self.norm_random:
                Q.synth_gaussian(buf.data_ptr(), d, self.seed + 4, 0.1)
                norm = (1.0 + buf[:d].cpu().numpy()).astype(np.float32)
            self._small = (router, bias, offset, norm)
        return self._small

    def build(self, torch, Q, dev, max_tokens, rank=0, world=1, nccl_id=None):
        """The layer on cuda:dev with its weights uploaded (an expert-parallel
        layer gets its own block of routed experts)."""
        c = self.cfg
        L = Q.MoeLayer(c["d_model"], c["n_experts"], c["n_active"], c["expert_ffn"],
                       moe_sigmoid=bool(c["moe_sigmoid"]), routed_scale=c["routed_scale"], n_shared=c["n_shared"],
                       swiglu_limit=c["swiglu_limit"], rms_eps=c["rms_eps"], fmt=self.fmt,
                       shared_fmt=self.fmt_sh if self.shared else self.fmt, device=dev, max_tokens=max_tokens,
                       rank=rank, world=world, nccl_id=nccl_id)
        self.upload_into(torch, Q, dev, L)
        return L

    def upload_into(self, torch, Q, dev, L):
        """Uploads this layer's weights into an existing layer L (a MoeLayer or
        a layer of a MoeStack) on cuda:dev."""
        first, count = L.expert_range()
        for e in range(first, first + count):
            for w in range(3):
                q, nb = self.synth_matrix(torch, Q, dev, e, w)
                L.upload_expert_device(e, w, self.fmt[w], q.data_ptr(), nb)
        if self.shared:
            for w in range(3):
                q, nb = self.synth_matrix(torch, Q, dev, -1, w)
                L.upload_expert_device(Q.SHARED_EXPERT, w, self.fmt_sh[w], q.data_ptr(), nb)
        router, bias, offset, norm = self.small_tensors(torch, Q, dev)
        L.upload_router(router, bias)
        if offset is not None:
            L.upload_logit_offset(offset)
        L.upload_norm(norm)
        torch.cuda.synchronize()

    # ---------------------------------------------------------------- oracle
    def oracle_case(self, torch, Q, dev, experts=None):
        """A tests.moe_case.MoeCase for the oracle holding host bytes of
        `experts` (all when None); the other slots hold zero bytes (the
        oracle never reads them unless routing selects them, which the
        routing check would report)."""
        c = self.cfg
        E = c["n_experts"]
        router, bias, offset, norm = self.small_tensors(torch, Q, dev)
        need = set(range(E)) if experts is None else set(int(e) for e in experts)
        zero = {w: np.zeros(Q.tensor_bytes(self.shape(w)[0] * self.shape(w)[1], self.qfmt[w]), np.uint8)
                for w in range(3)}
        mats = [[self.host_matrix(torch, Q, dev, e, w) if e in need else zero[w] for e in range(E)]
                for w in range(3)]
        shared = tuple(self.host_matrix(torch, Q, dev, -1, w) for w in range(3)) if self.shared else None
        return MoeCase(cfg=c, norm_w=norm, router=router, router_bias=bias, logit_offset=offset,
                       gate=mats[0], up=mats[1], down=mats[2], fmt_gate=self.fmt[0], fmt_up=self.fmt[1],
                       fmt_down=self.fmt[2], shared=shared, fmt_sh=self.fmt_sh)
