"""B200 verify target: a transformers Qwen3 model whose attention runs on the B200 kernels.

Mirrors ``PersistentQwenTarget`` (dspark_qwen/persistent_qwen_target.py:100-472):
requests own slots of a persistent KV store, ``verify`` runs one model forward over
the packed new tokens of several requests without touching committed KV,
``commit`` keeps each request's verified prefix (anchor included) and drops the
rest, ``prefill`` is verify + commit-all, ``predict`` applies the LM head, and
selected decoder outputs are captured as draft features.

The reference routes attention through an HF attention callback plus a Cache
subclass that stages K/V and gathers a capacity workspace every layer
(persistent_qwen_target.py:45-83). Here each layer's ``Qwen3Attention.forward``
is replaced by one that hands the raw q/k/v projections to the store:

* bf16 model: ``verify_layer`` — one fused kernel does q_norm/k_norm, RoPE, the
  KV append and bottom-right attention over the resident prefix;
* float32 model (exact path): transformers' own q_norm/k_norm/RoPE, then
  ``stage_layer`` + ``attend`` on the float32 attention kernel.

In a bf16 model the decoder layers' ``input_layernorm`` / ``post_attention_layernorm``
and the final ``norm`` also run as one ``rms_norm`` launch each instead of
transformers' eight-kernel sequence (the post-attention residual add and its norm as
one ``add_rms_norm``), each attention projects q, k and v with ONE GEMM
whose column blocks go to ``verify_layer`` as row-strided views, and each MLP projects
gate and up with ONE GEMM followed by ``silu_mul`` (the projection weights become views
of one merged buffer per layer and kind, values and memory unchanged). The float32 model keeps transformers'
modules.
"""
import types
from dataclasses import dataclass

import torch
from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

from .kernels import HEAD_DIM, HKV, HQ, add_rms_norm, merged_mlp_ready, rms_norm, silu_mul
from .kv_store import B200PersistentTargetKV


@dataclass
class TargetFeatures:
    last: torch.Tensor            # [1, sum Q, hidden] final-norm hidden states
    context: torch.Tensor | None  # [1, sum Q, len(layer_ids) * hidden] captured decoder outputs
    spans: dict                   # request -> (row offset, query rows, committed context before)
    work: dict

    def context_for(self, request):
        off, q, _ = self.spans[request]
        return self.context[:, off:off + q]


def _fused_norm_forward(norm, hidden_states):
    return rms_norm(hidden_states, norm.weight, norm.variance_epsilon)


def _decoder_layer_forward(layer, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                           use_cache=False, position_embeddings=None, **kwargs):
    """transformers' Qwen3DecoderLayer.forward with the post-attention residual add and
    ``post_attention_layernorm`` as one ``add_rms_norm`` launch (bf16)."""
    h = layer.input_layernorm(hidden_states)
    h, _ = layer.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                           past_key_values=past_key_values, use_cache=use_cache,
                           position_embeddings=position_embeddings, **kwargs)
    norm = layer.post_attention_layernorm
    residual, h = add_rms_norm(hidden_states, h, norm.weight, norm.variance_epsilon)
    return residual + layer.mlp(h)


def _merge_linears(linears):
    """One [out_1 + out_2 + ...; in] buffer holding the linears' weights; each weight
    becomes a view of its block (values unchanged)."""
    merged = torch.cat([lin.weight.detach() for lin in linears])
    off = 0
    for lin in linears:
        lin.weight.data = merged[off:off + lin.out_features]
        off += lin.out_features
    return merged


def _merged_mlp_forward(mlp):
    """Rebind gate_proj / up_proj weights as views of one merged buffer and return a
    forward that runs one GEMM, ``silu_mul`` and down_proj."""
    merged = _merge_linears((mlp.gate_proj, mlp.up_proj))
    inter = mlp.gate_proj.out_features

    def forward(m, x):
        return m.down_proj(silu_mul(torch.nn.functional.linear(x, merged), inter))
    return forward


class B200Qwen3Target:
    def __init__(self, model, layer_ids=(), *, slots, context_capacity, max_query_tokens, slot_capacities=None):
        config = model.config
        if (config.model_type != 'qwen3' or getattr(config, 'use_sliding_window', False)
                or any(kind != 'full_attention' for kind in config.layer_types)
                or config.rope_parameters.get('rope_type') != 'default'):
            raise ValueError('Dense Qwen3 with default RoPE required')
        if (config.num_attention_heads, config.num_key_value_heads, config.head_dim) != (HQ, HKV, HEAD_DIM):
            raise ValueError('B200 attention supports Hq16/Hkv8/D128 Qwen3 geometry')
        self.layer_ids = tuple(layer_ids)
        if (tuple(sorted(set(self.layer_ids))) != self.layer_ids
                or any(not 0 <= i < config.num_hidden_layers for i in self.layer_ids)):
            raise ValueError('Unique increasing valid decoder layer IDs required')
        weight = model.get_input_embeddings().weight
        if weight.device.type != 'cuda' or weight.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError('B200 target needs a bf16 (or exact-path float32) model on a CUDA device')
        self.model = model.eval().requires_grad_(False)
        self.dtype = weight.dtype
        self.pool = B200PersistentTargetKV(layers=config.num_hidden_layers, slots=slots,
                                           context_capacity=context_capacity, max_query_tokens=max_query_tokens,
                                           dtype=self.dtype, device=weight.device, slot_capacities=slot_capacities)
        self.inv_freq = model.model.rotary_emb.inv_freq.float().contiguous()
        self.eps = config.rms_norm_eps
        self._handles = {}
        self._tx = None
        self._pending = None
        self._captured = {}
        self._hooks = [model.model.layers[i].register_forward_hook(self._hook(i)) for i in self.layer_ids]
        self._graphs = {}
        self._orig_forward = {}
        self._qkv = {}
        for layer in model.model.layers:
            att = layer.self_attn
            self._orig_forward[att] = vars(att).get('forward')
            att.forward = types.MethodType(self._attention_forward(), att)
        if self.dtype == torch.bfloat16:
            norms = [m for layer in model.model.layers for m in (layer.input_layernorm, layer.post_attention_layernorm)]
            for norm in norms + [model.model.norm]:
                self._orig_forward[norm] = vars(norm).get('forward')
                norm.forward = types.MethodType(_fused_norm_forward, norm)
            for layer in model.model.layers:
                self._orig_forward[layer] = vars(layer).get('forward')
                layer.forward = types.MethodType(_decoder_layer_forward, layer)
                att = layer.self_attn
                if all(lin.bias is None for lin in (att.q_proj, att.k_proj, att.v_proj)):
                    self._qkv[att] = _merge_linears((att.q_proj, att.k_proj, att.v_proj))
                if merged_mlp_ready(layer.mlp):
                    self._orig_forward[layer.mlp] = vars(layer.mlp).get('forward')
                    layer.mlp.forward = types.MethodType(_merged_mlp_forward(layer.mlp), layer.mlp)

    @property
    def device(self):
        return self.pool.device

    @property
    def lengths(self):
        return {r: self.pool.length(h) for r, h in self._handles.items()}

    def _hook(self, index):
        def capture(_module, _inputs, output):
            if self._tx is None:
                raise RuntimeError('Foreign model forward while the B200 target owns the model')
            self._captured[index] = output[0] if isinstance(output, tuple) else output
        return capture

    def _attention_forward(self):
        target = self

        def forward(att, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None,
                    **kwargs):
            tx = target._tx
            if tx is None or hidden_states.shape[0] != 1:
                raise RuntimeError('B200 attention runs inside a verify transaction on one packed row')
            n = hidden_states.shape[1]
            merged = target._qkv.get(att)
            if merged is not None:                  # one GEMM; q/k/v are row-strided column blocks
                qkv = torch.nn.functional.linear(hidden_states, merged)[0]
                q = qkv[:, :HQ * HEAD_DIM].view(n, HQ, HEAD_DIM)
                k = qkv[:, HQ * HEAD_DIM:(HQ + HKV) * HEAD_DIM].view(n, HKV, HEAD_DIM)
                v = qkv[:, (HQ + HKV) * HEAD_DIM:].view(n, HKV, HEAD_DIM)
            else:
                q = att.q_proj(hidden_states).view(n, HQ, HEAD_DIM)
                k = att.k_proj(hidden_states).view(n, HKV, HEAD_DIM)
                v = att.v_proj(hidden_states).view(n, HKV, HEAD_DIM)
            if target.dtype == torch.bfloat16:
                out = target.pool.verify_layer(tx, att.layer_idx, q, k, v,
                                               att.q_norm.weight, att.k_norm.weight, inv_freq=target.inv_freq,
                                               eps=target.eps)
            else:
                cos, sin = position_embeddings
                qn = att.q_norm(q[None]).transpose(1, 2)
                kn = att.k_norm(k[None]).transpose(1, 2)
                qr, kr = apply_rotary_pos_emb(qn, kn, cos, sin)
                target.pool.stage_layer(tx, att.layer_idx, kr[0].transpose(0, 1).contiguous(), v.contiguous())
                out = target.pool.attend(tx, att.layer_idx, qr[0].transpose(0, 1).contiguous())
            return att.o_proj(out.reshape(1, n, -1)), None

        return forward

    # -- requests -------------------------------------------------------------------
    def add_request(self, request):
        if self._pending is not None:
            raise RuntimeError('Finish the outstanding verification first')
        handle = self.pool.add_request(request)
        self._handles[request] = handle
        return handle

    def remove_request(self, request):
        if self._pending is not None:
            raise RuntimeError('Finish the outstanding verification first')
        self.pool.remove_request(self._handles.pop(request))

    # -- verification transactions (persistent_qwen_target.py:389-457) ----------------
    @torch.no_grad()
    def verify(self, chunks):
        """chunks: ordered {request: ids [1, Q]}; committed KV is not modified."""
        if self._pending is not None:
            raise RuntimeError('Finish the outstanding verification first')
        if not chunks:
            raise ValueError('Nonempty ordered token mapping required')
        for request, ids in chunks.items():
            if request not in self._handles:
                raise ValueError('Request not resident')
            if (not isinstance(ids, torch.Tensor) or ids.ndim != 2 or ids.shape[0] != 1 or ids.shape[1] < 1
                    or ids.dtype != torch.long or ids.device != self.device):
                raise ValueError('Each token chunk must be [1,Q] long on the target device')
        handles = tuple(self._handles[r] for r in chunks)
        qlens = tuple(ids.shape[1] for ids in chunks.values())
        tx = self.pool.begin(handles, query_lengths=qlens)
        spans, offset, positions = {}, 0, []
        for request, c, q in zip(chunks, tx.context_lengths, qlens):
            spans[request] = (offset, q, c)
            positions.extend(range(c, c + q))
            offset += q
        pos = torch.tensor(positions, dtype=torch.long).pin_memory().to(self.device, non_blocking=True)
        self._tx, self._captured = tx, {}
        try:
            out = self.model.model(input_ids=torch.cat(tuple(chunks.values()), dim=1), position_ids=pos[None],
                                   attention_mask={'full_attention': None}, use_cache=False, return_dict=True)
            context = (torch.cat([self._captured[i] for i in self.layer_ids], dim=-1) if self.layer_ids else None)
            work = self.pool.work(tx)
            features = TargetFeatures(out.last_hidden_state, context, spans, work)
            self._pending = (features, tx)
            return features
        except BaseException:
            if self.pool._pending is tx and not self.pool.failed:
                self.pool.abort(tx)
            raise
        finally:
            self._tx, self._captured = None, {}

    # -- captured verify program (persistent_qwen_graph.py:198-275) --------------------
    def _forward(self, ids, pos):
        out = self.model.model(input_ids=ids, position_ids=pos, attention_mask={'full_attention': None},
                               use_cache=False, return_dict=True)
        context = torch.cat([self._captured[i] for i in self.layer_ids], dim=-1) if self.layer_ids else None
        return out.last_hidden_state, context

    @torch.no_grad()
    def capture(self, bucket):
        """Capture one full-model verify forward for ``bucket`` (exact ordered
        ``query_lengths``, e.g. the reference's ``Bucket``) into a CUDA graph. The
        program reads fixed-address token ids, positions and store metadata and writes
        fixed output buffers; ``verify_graph`` fills the inputs and replays it. As in
        the reference, metadata construction, sampling and commit stay outside."""
        if self._pending is not None:
            raise RuntimeError('Finish the outstanding verification first')
        if bucket in self._graphs:
            raise ValueError('Bucket already captured')
        n = sum(bucket.query_lengths)
        ids = torch.zeros((1, n), dtype=torch.long, device=self.device)
        pos = torch.zeros((1, n), dtype=torch.long, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):        # warm-up: library handles and allocator state
            tx = self.pool.capture_transaction(bucket)
            self._tx, self._captured = tx, {}
            try:
                self._forward(ids, pos)
            finally:
                self._tx, self._captured = None, {}
                self.pool.abort(tx)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        tx = self.pool.capture_transaction(bucket)
        self._tx, self._captured = tx, {}
        try:
            # captured on the warm-up stream, so the library workspace it binds is the
            # one allocated eagerly during warm-up
            with torch.cuda.graph(graph, stream=side):
                last, context = self._forward(ids, pos)
        finally:
            self._tx, self._captured = None, {}
            self.pool.abort(tx)
        self._graphs[bucket] = dict(graph=graph, ids=ids, pos=pos, last=last, context=context)
        return graph

    @torch.no_grad()
    def verify_graph(self, chunks, bucket):
        """``verify`` through the program captured for ``bucket``: the chunks' lengths
        must be the bucket's query lengths, in order. The returned features are views
        of the program's fixed output buffers, valid until the next replay."""
        if self._pending is not None:
            raise RuntimeError('Finish the outstanding verification first')
        ex = self._graphs.get(bucket)
        if ex is None:
            raise ValueError('Capture the bucket first')
        for request, ids in chunks.items():
            if request not in self._handles:
                raise ValueError('Request not resident')
            if (not isinstance(ids, torch.Tensor) or ids.ndim != 2 or ids.shape[0] != 1
                    or ids.dtype != torch.long or ids.device != self.device):
                raise ValueError('Each token chunk must be [1,Q] long on the target device')
        qlens = tuple(ids.shape[1] for ids in chunks.values())
        if qlens != tuple(bucket.query_lengths):
            raise ValueError('Chunk lengths differ from the captured bucket')
        tx = self.pool.begin(tuple(self._handles[r] for r in chunks), bucket)
        spans, offset, positions = {}, 0, []
        for request, c, q in zip(chunks, tx.context_lengths, qlens):
            spans[request] = (offset, q, c)
            positions.extend(range(c, c + q))
            offset += q
        ex['ids'].copy_(torch.cat(tuple(chunks.values()), dim=1))
        ex['pos'].copy_(torch.tensor([positions], dtype=torch.long).pin_memory(), non_blocking=True)
        ex['graph'].replay()
        self.pool.replayed(tx)
        features = TargetFeatures(ex['last'], ex['context'], spans, self.pool.work(tx))
        self._pending = (features, tx)
        return features

    @torch.no_grad()
    def commit(self, features, committed_query_lengths):
        """Keep each request's verified prefix (anchor included); the rest is rolled back."""
        if self._pending is None or self._pending[0] is not features:
            raise ValueError('Only the outstanding verification features can commit')
        if set(committed_query_lengths) != set(features.spans):
            raise ValueError('One committed query prefix per verified request required')
        _, tx = self._pending
        result = self.pool.commit(tx, {self._handles[r]: n for r, n in committed_query_lengths.items()})
        self._pending = None
        return result

    def abort(self, features):
        if self._pending is None or self._pending[0] is not features:
            raise ValueError('Only outstanding verification features can abort')
        self.pool.abort(self._pending[1])
        self._pending = None

    @torch.no_grad()
    def prefill(self, chunks):
        if any(r not in self._handles for r in chunks):
            raise ValueError('Request not resident')
        if any(self.pool.length(self._handles[r]) for r in chunks):
            raise ValueError('Prefill is only for newly admitted empty requests')
        features = self.verify(chunks)
        self.commit(features, {r: ids.shape[1] for r, ids in chunks.items()})
        return features

    @torch.no_grad()
    def predict(self, features, last_only=False):
        """LM head over the verified rows; {request: logits [1, Q|1, vocab]}."""
        logits = self.model.get_output_embeddings()(features.last)
        return {r: (logits[:, off + q - 1] if last_only else logits[:, off:off + q])
                for r, (off, q, _) in features.spans.items()}

    def close(self):
        """Restore the model's attention, norm and MLP forwards and release captured
        programs (merged gate/up weights stay views of their shared buffer)."""
        self._graphs.clear()
        for hook in self._hooks:
            hook.remove()
        for module, fwd in self._orig_forward.items():   # None: the class's forward was in use
            if fwd is None:
                del module.forward
            else:
                module.forward = fwd
        self._hooks, self._orig_forward = [], {}
