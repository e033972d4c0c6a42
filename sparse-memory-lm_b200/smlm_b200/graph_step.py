"""A whole training step captured as one CUDA graph (no counterpart in the reference).

A PKM training step is some sixty kernel launches driven from Python (autograd, the library's C calls, torch's
optimizers); on a busy host that driving can take longer than the GPU work. GraphedStep captures one step,
forward, backward, clipping and both optimizers, and replays it: per step the host copies the inputs into the
step's static buffers, advances the capturable optimizers (LazyRowAdam(capturable=True) writes its bias-correction
scalars; torch's capturable AdamW keeps its own step on the device) and launches the graph.

    step = GraphedStep(lambda x, g: train_step(mem, opt, x, g), [x0, g0], [lazy_adam], warmup=3)
    for x, g in batches:
        out = step(x, g)                 # the step's outputs (static tensors, valid until the next call)

Requirements: the same shapes every step, no host synchronisation inside the step, torch optimizers built with
capturable=True, LazyRowAdam(capturable=True) with fp32 moments (one backward per step takes the fused deferred step,
several the plain step over the written accumulator; both read their scalars from device memory). Build the
GraphedStep before running eager backward passes of the model on the legacy default stream: autograd ties each
parameter's gradient accumulation to the stream of its first backward, and the legacy stream cannot join a
capture (the warm-up steps here run on a side stream). Eager steps after the capture are fine.
"""
import torch


class GraphedStep:
    def __init__(self, step_fn, example_inputs, optimizers=(), warmup=3):
        """step_fn(*inputs) runs one step and returns a tensor or a tuple of tensors; example_inputs: device
        tensors of the inputs' shapes (their values are used for the warm-up steps); optimizers: the objects with
        a prepare_replay() method (LazyRowAdam(capturable=True)). The warm-up steps run eagerly: they are real
        training steps."""
        self.step_fn = step_fn
        self.static = [x.detach().clone() for x in example_inputs]
        self.optimizers = [o for o in optimizers if hasattr(o, "prepare_replay")]
        dev = self.static[0].device
        main = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                step_fn(*self.static)
        main.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = step_fn(*self.static)

    def __call__(self, *inputs, prepare=True):
        """One step: inputs copied into the static buffers (on the current stream), optimizers advanced, graph
        replayed. prepare=False when the caller advanced the optimizers itself."""
        for s, x in zip(self.static, inputs):
            if x is not s:
                s.copy_(x, non_blocking=True)
        if prepare:
            for o in self.optimizers:
                o.prepare_replay()
        self.graph.replay()
        return self.outputs
