"""Logic layers with the reference module API (``silogic/layers.py``), CUDA-only.

``LogicLayer`` = connectome + node; ``ConvLogicTree`` = a gate tree per output
channel over a k x k receptive field; ``OrPool`` = OR (max) pooling.  The
constructors, parameter names, buffers and seeded random draws follow the
reference so checkpoints load unchanged.  ``forward`` (soft, differentiable) and
``forward_hard`` (bit-packed Boolean circuit) run the sm_100a kernels of
``libsilogic_b200.so``; there is no CPU implementation.
"""
import torch
import torch.nn as nn

from . import _hard, _soft
from .connectomes import build_connectome, TopKConnectome, FixedConnectome, DenseConnectome
from .nodes import build_node, _NODE_ALIASES
from .functional import BASIS_COEFFS, TRUTH_TABLES, GATE_A


class LogicLayer(nn.Module):
    """A layer of logic nodes: connectome (input wiring) + node (gate parameterization).

    Same arguments as the reference ``LogicLayer`` (``silogic/layers.py:20-76``).
    ``use_triton`` is accepted for compatibility and ignored: the CUDA kernels
    are the only implementation.
    """

    def __init__(self, in_dim, out_dim, node="gate16", connectome="topk", arity=2,
                 k=8, gate_eval="basis", residual_p=0.0, seed=None,
                 window=0, tau=1.0, degree=None, gate_select="softmax",
                 gumbel_tau=1.0, use_triton=True):
        super().__init__()
        self._node_name = _NODE_ALIASES.get(str(node).lower(), node)
        if self._node_name == "gate16":
            arity = 2
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.arity = arity
        self.k = k
        self.gate_eval = gate_eval
        self.use_triton = use_triton
        self.connectome = connectome
        self._conn = build_connectome(connectome, in_dim, out_dim, arity, k, seed, window)
        if gate_select == "hard" and hasattr(self._conn, "ste"):
            self._conn.ste = True
        self.node = build_node(node, out_dim, arity, gate_eval=gate_eval, tau=tau,
                               degree=degree, gate_select=gate_select, gumbel_tau=gumbel_tau)
        if residual_p > 0:
            self.node.residual_init(residual_p)

    # compatibility accessors
    @property
    def gate_logits(self):
        return self.node.gate_logits

    @property
    def theta(self):
        return self.node.theta

    @property
    def conn_a(self):
        return self._conn.conn[:, 0]

    @property
    def conn_b(self):
        return self._conn.conn[:, 1]

    def _fused_ok(self, x):
        """True when ``forward`` runs the fused kernel (always, on CUDA)."""
        return x.is_cuda and _soft.fc_supported(self)

    def forward(self, x):
        return _soft.logic_layer_forward(self, x)

    @torch.no_grad()
    def hard_spec(self):
        """(wiring ``[out, arity]`` int32, truth tables ``[out]`` int64) on the param device."""
        idx = self._conn.hard_index().to(torch.int32).contiguous()
        tt = _hard.node_truth_tables(self.node.kind, self.node.param, self.arity,
                                     getattr(self.node, "mono_mask", None)).contiguous()
        return idx, tt

    @torch.no_grad()
    def forward_hard(self, x):
        B = x.shape[0]
        if x.reshape(B, -1).shape[1] != self.in_dim:
            raise ValueError(f"LogicLayer expects {self.in_dim} input features, got "
                             f"{x.reshape(B, -1).shape[1]}")
        idx, tt = self.hard_spec()
        _hard.check_index_range(idx, self.in_dim, "LogicLayer wiring")
        return _hard.unpack(_hard.fc(_hard.pack(x), idx, tt), B)


class WARPLayer(LogicLayer):
    """2-input Walsh (WARP) node with Top-K connectivity."""

    def __init__(self, in_dim, out_dim, k=8, tau=1.0, residual_p=0.0, seed=None,
                 gate_select="softmax"):
        super().__init__(in_dim, out_dim, node="walsh", connectome="topk", arity=2, k=k,
                         tau=tau, residual_p=residual_p, seed=seed, gate_select=gate_select)

    @property
    def theta(self):
        return self.node.theta

    def _z(self, a, b):
        return self.node._z(a, b)

    def _coef(self):
        return self.node.coef()


class WARPLayerN(LogicLayer):
    """Arity-n Walsh node with Top-K connectivity."""

    def __init__(self, in_dim, out_dim, arity=6, k=8, tau=1.0, residual_p=0.0, seed=None,
                 gate_select="softmax"):
        super().__init__(in_dim, out_dim, node="walsh", connectome="topk", arity=arity, k=k,
                         tau=tau, residual_p=residual_p, seed=seed, gate_select=gate_select)

    @property
    def theta(self):
        return self.node.theta


class LUTkLayer(LogicLayer):
    """k-input multilinear LUT node with Top-K (or fixed) input selection."""

    def __init__(self, in_dim, out_dim, k=4, learn_conn=True, cand_k=4, seed=None):
        super().__init__(in_dim, out_dim, node="multilinear",
                         connectome="topk" if learn_conn else "fixed", arity=k, k=cand_k,
                         seed=seed)
        self.k = k
        self.learn_conn = learn_conn

    @property
    def lut(self):
        return self.node.logits

    @property
    def conn(self):
        return self._conn.conn

    @property
    def cand(self):
        return self._conn.cand


class LUTNodeLayer(LogicLayer):
    """n-input LUT node with a selectable relaxation."""

    def __init__(self, in_dim, out_dim, arity=4, relaxation="probabilistic", k=8,
                 degree=None, residual_p=0.0, seed=None):
        super().__init__(in_dim, out_dim, node=relaxation, connectome="topk", arity=arity,
                         k=k, degree=degree, residual_p=residual_p, seed=seed)
        self.relaxation = relaxation
        self.n = arity
        self.k = self._conn.k

    @property
    def conn(self):
        return self._conn.conn

    @property
    def cand(self):
        return self._conn.cand


class ConvLogicTree(nn.Module):
    """Logic-gate-tree convolution (a node tree per output channel over a k x k field).

    Same arguments, buffers and seeded draws as the reference
    (``silogic/layers.py:226-365``).  ``forward`` returns ``[B, n, Ho, Wo]``;
    inside :class:`~silogic_b200.models.LogicConvNet` the following ``OrPool`` is
    fused into the same kernel.
    """

    def __init__(self, in_channels, out_channels, kernel=3, tree_depth=None, stride=1,
                 padding=1, connect="topk", k=4, n_chan=2, residual_init=True, seed=0,
                 node="gate16", arity=4, tau=1.0, degree=None, gate_select="softmax",
                 gumbel_tau=1.0, use_triton=True):
        super().__init__()
        self.node_name = _NODE_ALIASES.get(str(node).lower(), node)
        self.gate_select = gate_select
        self.gumbel_tau = gumbel_tau
        self.node_arity = 2 if self.node_name in ("gate16", "walsh") else arity
        if tree_depth is None:
            tree_depth = 2 if self.node_arity == 2 else 1
        self.cin = in_channels
        self.n = out_channels
        self.kh = self.kw = kernel
        self.d = tree_depth
        self.leaves = self.node_arity ** tree_depth
        self.stride = stride
        self.padding = padding
        self.connect = connect
        self.k = k
        self.tau = tau
        self.use_triton = use_triton
        gen = torch.Generator().manual_seed(seed)

        kk2 = kernel * kernel
        pool_sz = n_chan * kk2
        pools = []
        for _ in range(out_channels):                     # n_chan random channels per tree
            chans = torch.randperm(in_channels, generator=gen)[:n_chan]
            taps = []
            for c in chans:
                taps.extend(range(int(c) * kk2, int(c) * kk2 + kk2))
            pools.append(torch.tensor(taps))
        pools = torch.stack(pools)                        # [n, pool_sz]
        if connect == "fixed":
            sel = torch.stack([pools[i][torch.randint(0, pool_sz, (self.leaves,), generator=gen)]
                               for i in range(out_channels)])
            self.register_buffer("leaf_idx", sel)
            self.register_buffer("cm_idx", (sel // kk2).to(torch.int32))
            self.register_buffer("ch_idx", ((sel % kk2) // kernel).to(torch.int32))
            self.register_buffer("cw_idx", ((sel % kk2) % kernel).to(torch.int32))
        else:
            kk = min(k, pool_sz)
            self.k = kk
            cand = torch.stack([
                torch.stack([pools[i][torch.randperm(pool_sz, generator=gen)[:kk]]
                             for _ in range(self.leaves)]) for i in range(out_channels)])
            self.register_buffer("leaf_cand", cand)
            self.conn = nn.Parameter(torch.randn(out_channels, self.leaves, kk))
            self.register_buffer("lc_cm", (cand // kk2).to(torch.int32))
            self.register_buffer("lc_ch", ((cand % kk2) // kernel).to(torch.int32))
            self.register_buffer("lc_cw", ((cand % kk2) % kernel).to(torch.int32))

        if self.node_name == "gate16":
            self.gate_logits = nn.ParameterList()
            for i in range(tree_depth):
                w = torch.zeros(out_channels, 2 ** (tree_depth - 1 - i), 16)
                if residual_init:
                    w[:, :, GATE_A] = 5.0
                else:
                    w.normal_(0, 0.1)
                self.gate_logits.append(nn.Parameter(w))
            self.register_buffer("basis", BASIS_COEFFS.clone())
            self.register_buffer("truth", TRUTH_TABLES.clone())
        else:
            self.tree_nodes = nn.ModuleList()
            for i in range(tree_depth):
                m = self.node_arity ** (tree_depth - 1 - i)
                nd = build_node(self.node_name, out_channels * m, arity=self.node_arity,
                                tau=tau, degree=degree, gate_select=gate_select,
                                gumbel_tau=gumbel_tau)
                if residual_init:
                    nd.residual_init(0.9)
                self.tree_nodes.append(nd)

    @property
    def gates_per_output(self):
        k = self.node_arity
        return (k ** self.d - 1) // (k - 1)

    def _hw_out(self, H, W):
        Ho = (H + 2 * self.padding - self.kh) // self.stride + 1
        Wo = (W + 2 * self.padding - self.kw) // self.stride + 1
        return Ho, Wo

    def level_params(self):
        """Per-level parameter tensors: gate logits ``[n, nodes, 16]`` or node params."""
        if self.node_name == "gate16":
            return list(self.gate_logits)
        return [nd.param for nd in self.tree_nodes]

    @torch.no_grad()
    def hard_leaves(self):
        """Hard-selected receptive-field tap per (channel, leaf): ``[n, leaves]`` int32."""
        if self.connect == "fixed":
            sel = self.leaf_idx
        else:
            sel = torch.gather(self.leaf_cand, 2, self.conn.argmax(dim=2).unsqueeze(-1)).squeeze(-1)
        return sel.to(torch.int32).contiguous()

    @torch.no_grad()
    def hard_spec(self):
        """(leaves ``[n, leaves]`` int32, truth tables ``[n, total_nodes]`` int64, level 0 first)."""
        tts = []
        for i, prm in enumerate(self.level_params()):
            m = self.node_arity ** (self.d - 1 - i)
            if self.node_name == "gate16":
                t = _hard.node_truth_tables("gate16", prm, 2)            # [n, m]
            else:
                nd = self.tree_nodes[i]
                t = _hard.node_truth_tables(nd.kind, prm, self.node_arity,
                                            getattr(nd, "mono_mask", None)).view(self.n, m)
            tts.append(t)
        return self.hard_leaves(), torch.cat(tts, dim=1).contiguous()

    def forward(self, x):
        return _soft.conv_tree_forward(self, x, pool=1)

    @torch.no_grad()
    def forward_hard(self, x):
        B, C, H, W = x.shape
        if C != self.cin:
            raise ValueError(f"ConvLogicTree expects {self.cin} input channels, got {C}")
        leaf, tt = self.hard_spec()
        _hard.check_index_range(leaf, self.cin * self.kh * self.kw, "ConvLogicTree leaf taps")
        h = _hard.pack(x.reshape(B, -1)).view(C, H, W, -1)
        y = _hard.conv(h, leaf, tt, self.node_arity, self.d, self.kh, self.padding, pool=1)
        Ho, Wo = self._hw_out(H, W)
        return _hard.unpack(y.view(-1, y.shape[-1]), B).view(B, self.n, Ho, Wo)


ConvLogicLayer = ConvLogicTree


class OrPool(nn.Module):
    """OR pooling (max t-conorm): ``size x size`` window and stride."""

    def __init__(self, size=2):
        super().__init__()
        self.size = size

    def forward(self, x):
        return _soft.or_pool(x, self.size)

    @torch.no_grad()
    def forward_hard(self, x):
        return _soft.or_pool_hard(x, self.size)
