"""Training and evaluation with the API of ``silogic/train.py`` (``eval_hard``,
``eval_soft``, ``train_model``), built for the CUDA kernels of this package.

Where the reference wraps the model in ``torch.compile`` (``train.py:125``), a training step
here -- the on-device augmentation (bit flips, cutout), the fused soft forward and backward
kernels, the cross-entropy and an Adam/AdamW step with ``capturable=True`` -- is captured
once as a CUDA graph over static batch buffers and replayed for every batch: one launch per
step instead of a few hundred, with the batch gathered on the device into the static input.
``graph=False`` runs the same step eagerly.  ``compile_`` is accepted for signature parity.
"""
import functools
import math
import time

import torch
import torch.nn.functional as F

_print = functools.partial(print, flush=True)


@torch.no_grad()
def eval_hard(model, X, y, device, bs=1024):
    """Top-1 accuracy (%) of the hard Boolean circuit (``train.py:15-37``): the bit-packed
    plan is built once and every batch runs pack -> layers -> GroupSum on the GPU."""
    from .bitpacking.plan import HardPlan
    model.eval()
    plan = HardPlan.from_model(model.to(device))
    correct = 0
    for i in range(0, X.shape[0], bs):
        xb = X[i:i + bs].to(device)
        pred = plan.counts(xb).argmax(dim=1).cpu()
        correct += (pred == y[i:i + bs]).sum().item()
    return 100.0 * correct / X.shape[0]


@torch.no_grad()
def eval_soft(model, X, y, device, bs=1024):
    """Top-1 accuracy (%) of the soft forward (``train.py:40-60``)."""
    model.eval()
    correct = 0
    for i in range(0, X.shape[0], bs):
        logits = model(X[i:i + bs].to(device).float())
        correct += (logits.argmax(dim=1).cpu() == y[i:i + bs]).sum().item()
    return 100.0 * correct / X.shape[0]


def _augment(xb, flip_p, cutout):
    """Bit-flip and cutout augmentation on the device (``train.py:150-163``)."""
    if flip_p > 0.0:
        m = torch.rand_like(xb) < flip_p
        xb = torch.where(m, 1.0 - xb, xb)
    if cutout > 0 and xb.dim() == 4:
        B, _, H, W = xb.shape
        cy = torch.randint(0, H, (B,), device=xb.device)
        cx = torch.randint(0, W, (B,), device=xb.device)
        yy = torch.arange(H, device=xb.device).view(1, H, 1)
        xx = torch.arange(W, device=xb.device).view(1, 1, W)
        r = cutout // 2
        mask = (((yy - cy.view(B, 1, 1)).abs() <= r) &
                ((xx - cx.view(B, 1, 1)).abs() <= r)).unsqueeze(1)
        xb = xb.masked_fill(mask, 0.0)
    return xb


class GraphedTrainStep:
    """One training step over static batch buffers, captured as a CUDA graph.

    ``step(x_u8, y)`` copies the batch into the static buffers and runs the step: the
    first ``warmup`` calls run it eagerly on a side stream (real steps on real batches,
    which also settle the allocator and every lazily built buffer), the next call captures
    it, and every later call replays the graph.  ``loss`` is the last step's loss on the
    device.  The optimizer must be built with ``capturable=True`` so that its step counter
    and learning rate live on the device.
    """

    def __init__(self, model, opt, x_shape, device, flip_p=0.0, cutout=0, warmup=3):
        self.model, self.opt, self.device = model, opt, device
        self.x = torch.zeros(x_shape, dtype=torch.uint8, device=device)
        self.y = torch.zeros(x_shape[0], dtype=torch.int64, device=device)
        self.flip_p, self.cutout, self.warmup = flip_p, cutout, warmup
        self.graph, self.loss, self.done = None, None, 0

    def _body(self):
        xb = _augment(self.x.float(), self.flip_p, self.cutout)
        loss = F.cross_entropy(self.model(xb), self.y)
        self.opt.zero_grad(set_to_none=False)
        loss.backward()
        self.opt.step()
        return loss.detach()        # keep no autograd graph alive between steps

    def step(self, xb, yb):
        self.x.copy_(xb, non_blocking=True)
        self.y.copy_(yb, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            return self.loss
        main = torch.cuda.current_stream(self.device)
        if self.done < self.warmup:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                loss = self._body()
            main.wait_stream(side)
            self.done += 1
            return loss
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):          # recorded, not run
            self.loss = self._body()
        self.graph.replay()
        return self.loss


def train_model(model, Xtr, ytr, Xte, yte, device, epochs=200, bs=256, lr=0.075,
                val_every=25, gpu_data=True, log=_print, Xval=None, yval=None, compile_=True,
                eval_bs=1024, optimizer="adam", weight_decay=0.0, cosine=False, flip_p=0.0,
                cutout=0, graph=True):
    """Train and return ``{"test_soft", "test_hard", "train_min", "history"}``
    (``train.py:63-193``; same arguments and results).  ``Xtr`` / ``Xte`` are uint8;
    batches are static (``drop_last``), so every step replays the captured graph."""
    if not str(device).startswith("cuda"):
        raise RuntimeError("silogic_b200 trains on CUDA only (no CPU implementation)")
    model.to(device)
    params = list(model.parameters())
    # a captured step reads the learning rate from the device, so cosine decay still applies
    kw = dict(lr=torch.tensor(float(lr), device=device) if graph else lr, capturable=bool(graph))
    if optimizer == "adamw":
        opt = torch.optim.AdamW(params, weight_decay=weight_decay, **kw)
    else:
        opt = torch.optim.Adam(params, **kw)
    n = Xtr.shape[0]
    if gpu_data:
        try:
            Xtr_d, ytr_d = Xtr.to(device), ytr.to(device)
        except RuntimeError:
            gpu_data = False
    if not gpu_data:
        Xtr_d, ytr_d = Xtr, ytr
    nb = n // bs
    model.train()
    stepper = None
    if graph and nb > 0:
        stepper = GraphedTrainStep(model, opt, (bs,) + tuple(Xtr.shape[1:]), device, flip_p, cutout)

    history = {"val_acc": [], "bin_val_acc": [], "epoch": []}
    loss = torch.zeros((), device=device)
    t0 = time.time()
    for ep in range(epochs):
        model.train()
        if cosine:
            cur = 0.5 * lr * (1 + math.cos(math.pi * ep / epochs))
            for g in opt.param_groups:
                if torch.is_tensor(g["lr"]):
                    g["lr"].fill_(cur)
                else:
                    g["lr"] = cur
        perm = torch.randperm(n, device=device if gpu_data else "cpu")
        for b in range(nb):
            bidx = perm[b * bs:(b + 1) * bs]
            xb = Xtr_d[bidx].to(device, non_blocking=True)
            yb = ytr_d[bidx].to(device, non_blocking=True)
            if stepper is not None:
                loss = stepper.step(xb, yb)
            else:
                xf = _augment(xb.float(), flip_p, cutout)
                loss = F.cross_entropy(model(xf), yb)
                opt.zero_grad()
                loss.backward()
                opt.step()
                loss = loss.detach()
        if (ep + 1) % val_every == 0 or ep == epochs - 1:
            Xv = Xval if Xval is not None else Xte
            yv = yval if yval is not None else yte
            va = eval_soft(model, Xv, yv, device, bs=eval_bs)
            ba = eval_hard(model, Xv, yv, device, bs=eval_bs)
            history["epoch"].append(ep + 1)
            history["val_acc"].append(va)
            history["bin_val_acc"].append(ba)
            log(f"  epoch {ep + 1:3d}  loss {loss.item():.4f}  soft {va:.2f}  hard {ba:.2f}  "
                f"[{(time.time() - t0) / 60:.1f} min]")
    train_min = (time.time() - t0) / 60.0
    return {"test_soft": eval_soft(model, Xte, yte, device, bs=eval_bs),
            "test_hard": eval_hard(model, Xte, yte, device, bs=eval_bs),
            "train_min": train_min, "history": history}
