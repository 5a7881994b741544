using System.Collections.Concurrent;
using System.Text;
using ProjectAI.Core;

namespace ProjectAI.Backends.Cuda;

/// <summary>
/// The storage behind <see cref="Tensor.Handle"/> for tensors of a <see cref="CudaComputeBackend"/>: the device base
/// pointer of one allocator block. Views share the handle object (Tensor.cs:55-168 rewrite only shape, strides and
/// offset), so the block lives as long as any view of it does, or until the scope that owns it ends.
/// </summary>
internal sealed class CudaBuffer
{
    internal CudaBuffer(CudaComputeBackend owner, IntPtr @base, int scope)
    {
        Owner = owner;
        Base = @base;
        Scope = scope;
    }

    internal CudaComputeBackend Owner { get; }
    internal IntPtr Base { get; }

    /// <summary>Index of the open scope that owns the block, or -1 when no scope does.</summary>
    internal int Scope { get; set; }

    /// <summary>True once the native side has freed the block (its scope ended, Release, or a finalized view).</summary>
    internal bool Freed { get; set; }

    // The garbage collector's thread must not call into CUDA: the block is queued and freed by the next call on the
    // backend (CudaComputeBackend.Drain), under the backend's lock.
    ~CudaBuffer()
    {
        if (!Freed) Owner.EnqueueFinalized(this);
    }
}

/// <summary>
/// <see cref="IComputeBackend"/> on a B200 (sm_100a) through libprojectai_cuda.so (include/projectai_cuda.h).
/// Every op forwards to one C entry point: the inputs go down as view descriptors (base, element offset, dims,
/// element strides), the result comes back as a fresh contiguous block wrapped in a new <see cref="Tensor"/>.
/// All work is ordered on the context's CUDA stream; only <see cref="ToHost"/> (and the ops the library documents
/// as returning host values) wait for the device.
///
/// <para>Lifetime follows the seam's contract (IComputeBackend.cs:69-95) with the semantics of
/// TorchComputeBackend.cs:208-218: a block created inside a scope is freed when the scope is disposed unless
/// <see cref="KeepAlive"/> moved it exactly one level out; <see cref="Release"/> frees at once; a block no scope owns
/// is freed when its last view is collected. The backend mirrors the library's scope ownership per block, so a
/// finalizer never frees an address the allocator has already handed to a newer tensor.</para>
///
/// <para>Threading: one context, one stream. Calls are serialised by a lock; the library sets the device for the
/// calling thread on every entry, so the server's thread-pool threads (ComputeRegistry.cs:11) may call in.</para>
/// </summary>
public sealed unsafe class CudaComputeBackend : IComputeBackend
{
    private IntPtr _ctx;
    private readonly object _gate = new();
    private readonly List<HashSet<CudaBuffer>> _scopes = new();
    private readonly ConcurrentQueue<CudaBuffer> _finalized = new();

    public CudaComputeBackend(int device = 0)
    {
        IntPtr ctx;
        Native.Check(Native.CtxCreate(device, &ctx));
        _ctx = ctx;
        Device = new Device(DeviceKind.Cuda, device);
        byte* buf = stackalloc byte[128];
        Native.Check(Native.DeviceName(_ctx, buf, 128));
        DeviceName = Encoding.UTF8.GetString(buf, IndexOfZero(buf, 128));
    }

    public string Name => "cuda-b200";
    public Device Device { get; }

    /// <summary>The CUDA device's name, e.g. "NVIDIA B200".</summary>
    public string DeviceName { get; }

    /// <summary>True when the backend offers the fused extensions (the optional hooks of the seam).</summary>
    public bool SupportsFusedOps => true;

    /// <summary>
    /// Probes whether the backend can run on this machine: the library loads and a context can be created on
    /// device 0 (an sm_100 GPU; the library refuses other devices). Never throws, like
    /// TorchComputeBackend.IsAvailable (TorchComputeBackend.cs:42-74).
    /// </summary>
    public static bool IsAvailable(out string? reason)
    {
        try
        {
            IntPtr ctx;
            int st = Native.CtxCreate(0, &ctx);
            if (st != 0)
            {
                reason = Native.LastMessage();
                return false;
            }
            Native.CtxDestroy(ctx);
            reason = null;
            return true;
        }
        catch (Exception ex) when (ex is DllNotFoundException or EntryPointNotFoundException or BadImageFormatException)
        {
            reason = $"libprojectai_cuda.so not loadable ({ex.Message})";
            return false;
        }
    }

    // ------------------------------------------------------------ Allocation & host transfer (IComputeBackend.cs:15-18)

    public Tensor Allocate(Shape shape, DType dtype)
    {
        lock (_gate)
        {
            Drain();
            int* dims = stackalloc int[PaiTensor.MaxRank];
            int rank = Dims(shape, dims);
            PaiTensor o;
            Native.Check(Native.Alloc(Ctx, rank, dims, (int)dtype, &o));
            return Wrap(o);
        }
    }

    public Tensor FromHost(ReadOnlySpan<float> data, Shape shape, DType dtype)
    {
        lock (_gate)
        {
            Drain();
            int* dims = stackalloc int[PaiTensor.MaxRank];
            int rank = Dims(shape, dims);
            PaiTensor o;
            fixed (float* p = data) Native.Check(Native.FromHost(Ctx, p, data.Length, rank, dims, (int)dtype, &o));
            return Wrap(o);
        }
    }

    public void ToHost(Tensor source, Span<float> destination)
    {
        lock (_gate)
        {
            Drain();
            var s = Desc(source);
            fixed (float* p = destination) Native.Check(Native.ToHost(Ctx, &s, p, destination.Length));
        }
    }

    public void Copy(Tensor source, Tensor destination)
    {
        lock (_gate)
        {
            Drain();
            var s = Desc(source);
            var d = Desc(destination);
            Native.Check(Native.Copy(Ctx, &s, &d));
        }
    }

    // ------------------------------------------------------------ Elementwise (IComputeBackend.cs:20-31)

    public Tensor Add(Tensor a, Tensor b) => Binary(a, b, 0);
    public Tensor Mul(Tensor a, Tensor b) => Binary(a, b, 1);
    public Tensor Sub(Tensor a, Tensor b) => Binary(a, b, 2);
    public Tensor Div(Tensor a, Tensor b) => Binary(a, b, 3);

    public Tensor AddScalar(Tensor a, float scalar)
    {
        lock (_gate)
        {
            Drain();
            var x = Desc(a);
            PaiTensor o;
            Native.Check(Native.AddScalar(Ctx, &x, scalar, &o));
            return Wrap(o);
        }
    }

    public Tensor MulScalar(Tensor a, float scalar)
    {
        lock (_gate)
        {
            Drain();
            var x = Desc(a);
            PaiTensor o;
            Native.Check(Native.MulScalar(Ctx, &x, scalar, &o));
            return Wrap(o);
        }
    }

    public Tensor Sqrt(Tensor x) => Unary(x, 0);
    public Tensor Sigmoid(Tensor x) => Unary(x, 1);

    // ------------------------------------------------------------ Linear algebra (IComputeBackend.cs:33-35)

    public Tensor MatMul(Tensor a, Tensor b, bool transposeB = false)
    {
        lock (_gate)
        {
            Drain();
            var x = Desc(a);
            var y = Desc(b);
            PaiTensor o;
            Native.Check(Native.MatMul(Ctx, &x, &y, transposeB ? 1 : 0, &o));
            return Wrap(o);
        }
    }

    // ------------------------------------------------------------ Reductions (IComputeBackend.cs:37-43)

    public Tensor Sum(Tensor x, int axis, bool keepDims = false) => Reduce(x, axis, keepDims, 0);
    public Tensor Mean(Tensor x, int axis, bool keepDims = false) => Reduce(x, axis, keepDims, 1);
    public Tensor Max(Tensor x, int axis, bool keepDims = false) => Reduce(x, axis, keepDims, 2);

    // ------------------------------------------------------------ Transformer primitives (IComputeBackend.cs:45-49)

    public Tensor Softmax(Tensor x, int axis)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            PaiTensor o;
            Native.Check(Native.Softmax(Ctx, &d, axis, &o));
            return Wrap(o);
        }
    }

    public Tensor RmsNorm(Tensor x, Tensor weight, float eps)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            var w = Desc(weight);
            PaiTensor o;
            Native.Check(Native.RmsNorm(Ctx, &d, &w, eps, &o));
            return Wrap(o);
        }
    }

    public Tensor Silu(Tensor x) => Unary(x, 2);

    public Tensor RotaryEmbedding(Tensor x, Tensor cos, Tensor sin)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            var c = Desc(cos);
            var s = Desc(sin);
            PaiTensor o;
            Native.Check(Native.Rotary(Ctx, &d, &c, &s, &o));
            return Wrap(o);
        }
    }

    // ------------------------------------------------------------ Indexing & loss (IComputeBackend.cs:51-59)

    public Tensor Gather(Tensor table, int[] ids)
    {
        lock (_gate)
        {
            Drain();
            var t = Desc(table);
            PaiTensor o;
            fixed (int* p = ids) Native.Check(Native.Gather(Ctx, &t, p, ids.Length, &o));
            return Wrap(o);
        }
    }

    public Tensor ScatterAddRows(Tensor rows, int[] ids, int rowCount)
    {
        lock (_gate)
        {
            Drain();
            var r = Desc(rows);
            PaiTensor o;
            fixed (int* p = ids) Native.Check(Native.ScatterAddRows(Ctx, &r, p, ids.Length, rowCount, &o));
            return Wrap(o);
        }
    }

    public Tensor CrossEntropy(Tensor logits, int[] targets, int ignoreIndex)
    {
        lock (_gate)
        {
            Drain();
            var l = Desc(logits);
            PaiTensor o;
            fixed (int* p = targets) Native.Check(Native.CrossEntropy(Ctx, &l, p, targets.Length, ignoreIndex, &o));
            return Wrap(o);
        }
    }

    public Tensor CrossEntropyGrad(Tensor logits, int[] targets, int ignoreIndex)
    {
        lock (_gate)
        {
            Drain();
            var l = Desc(logits);
            PaiTensor o;
            fixed (int* p = targets) Native.Check(Native.CrossEntropyGrad(Ctx, &l, p, targets.Length, ignoreIndex, &o));
            return Wrap(o);
        }
    }

    // ------------------------------------------------------------ Structural (IComputeBackend.cs:61-68)

    public Tensor Cat(Tensor a, Tensor b, int axis)
    {
        lock (_gate)
        {
            Drain();
            var x = Desc(a);
            var y = Desc(b);
            PaiTensor o;
            Native.Check(Native.Cat(Ctx, &x, &y, axis, &o));
            return Wrap(o);
        }
    }

    // ------------------------------------------------------------ Scopes (IComputeBackend.cs:69-95)

    public IDisposable BeginScope()
    {
        lock (_gate)
        {
            Drain();
            Native.Check(Native.ScopeBegin(Ctx));
            _scopes.Add(new HashSet<CudaBuffer>());
            return new ScopeHandle(this, _scopes.Count);
        }
    }

    public void KeepAlive(Tensor tensor)
    {
        lock (_gate)
        {
            Drain();
            var buf = Buffer(tensor);
            if (buf.Freed) throw new InvalidOperationException("KeepAlive of a released tensor");
            Native.Check(Native.KeepAlive(Ctx, buf.Base));
            if (buf.Scope < 0) return;
            _scopes[buf.Scope].Remove(buf);
            buf.Scope -= 1;  // exactly one level out (IComputeBackend.cs:80-87)
            if (buf.Scope >= 0) _scopes[buf.Scope].Add(buf);
        }
    }

    public void Release(Tensor tensor)
    {
        lock (_gate)
        {
            Drain();
            var buf = Buffer(tensor);
            if (!buf.Freed) Free(buf);
        }
    }

    public void Dispose()
    {
        lock (_gate)
        {
            if (_ctx == IntPtr.Zero) return;
            foreach (var scope in _scopes)
                foreach (var b in scope) b.Freed = true;
            _scopes.Clear();
            Native.Check(Native.CtxDestroy(_ctx));
            _ctx = IntPtr.Zero;
        }
        GC.SuppressFinalize(this);
    }

    private sealed class ScopeHandle : IDisposable
    {
        private readonly CudaComputeBackend _owner;
        private readonly int _depth;
        private bool _done;

        internal ScopeHandle(CudaComputeBackend owner, int depth)
        {
            _owner = owner;
            _depth = depth;
        }

        public void Dispose()
        {
            if (_done) return;
            _done = true;
            _owner.EndScope(_depth);
        }
    }

    private void EndScope(int depth)
    {
        lock (_gate)
        {
            if (_scopes.Count != depth) throw new InvalidOperationException("scopes must be disposed innermost first");
            var owned = _scopes[^1];
            _scopes.RemoveAt(_scopes.Count - 1);
            foreach (var b in owned) b.Freed = true;  // the native scope frees their blocks
            Native.Check(Native.ScopeEnd(Ctx));
        }
    }

    // ------------------------------------------------------------ Fused extensions (optional hooks of the seam)
    // Each replaces a composed chain of the reference; a caller that does not find the hook composes the chain.

    /// <summary>Causal GQA attention (Modules.cs:169-196): output [B,S,H,D] and row log-sum-exp [B,H,S].</summary>
    public (Tensor Output, Tensor Lse) ScaledDotProductAttention(Tensor q, Tensor k, Tensor v, float scale, bool causal,
                                                                 int posOffset)
    {
        lock (_gate)
        {
            Drain();
            var dq = Desc(q);
            var dk = Desc(k);
            var dv = Desc(v);
            PaiTensor o, l;
            Native.Check(Native.SdpaFwd(Ctx, &dq, &dk, &dv, scale, causal ? 1 : 0, posOffset, &o, &l));
            return (Wrap(o), Wrap(l));
        }
    }

    /// <summary>Gradients of <see cref="ScaledDotProductAttention"/> (Autograd.cs:54-73 and :197-205 fused).</summary>
    public (Tensor Dq, Tensor Dk, Tensor Dv) ScaledDotProductAttentionBackward(Tensor q, Tensor k, Tensor v,
                                                                              Tensor output, Tensor lse, Tensor dOutput,
                                                                              float scale, bool causal, int posOffset)
    {
        lock (_gate)
        {
            Drain();
            var dq = Desc(q);
            var dk = Desc(k);
            var dv = Desc(v);
            var o = Desc(output);
            var l = Desc(lse);
            var g = Desc(dOutput);
            PaiTensor rq, rk, rv;
            Native.Check(Native.SdpaBwd(Ctx, &dq, &dk, &dv, &o, &l, &g, scale, causal ? 1 : 0, posOffset, &rq, &rk, &rv));
            return (Wrap(rq), Wrap(rk), Wrap(rv));
        }
    }

    /// <summary>RMSNorm backward (Autograd.cs:223-244) in one pass over x and the upstream gradient.</summary>
    public (Tensor Dx, Tensor Dw) RmsNormBackward(Tensor x, Tensor weight, Tensor grad, float eps)
    {
        lock (_gate)
        {
            Drain();
            var dx = Desc(x);
            var w = Desc(weight);
            var g = Desc(grad);
            PaiTensor rx, rw;
            Native.Check(Native.RmsNormBwd(Ctx, &dx, &w, &g, eps, &rx, &rw));
            return (Wrap(rx), Wrap(rw));
        }
    }

    /// <summary>silu(gate) ⊙ up (SwiGluFeedForward, Modules.cs:103-108).</summary>
    public Tensor SiluMul(Tensor gate, Tensor up)
    {
        lock (_gate)
        {
            Drain();
            var a = Desc(gate);
            var b = Desc(up);
            PaiTensor o;
            Native.Check(Native.SiluMulFwd(Ctx, &a, &b, &o));
            return Wrap(o);
        }
    }

    public (Tensor DGate, Tensor DUp) SiluMulBackward(Tensor gate, Tensor up, Tensor grad)
    {
        lock (_gate)
        {
            Drain();
            var a = Desc(gate);
            var b = Desc(up);
            var g = Desc(grad);
            PaiTensor ra, rb;
            Native.Check(Native.SiluMulBwd(Ctx, &a, &b, &g, &ra, &rb));
            return (Wrap(ra), Wrap(rb));
        }
    }

    /// <summary>Cross-entropy and its gradient (scaled by gradScale) in one read of the logits (Autograd.cs:187-192).</summary>
    public (Tensor Loss, Tensor Grad) CrossEntropyWithGrad(Tensor logits, int[] targets, int ignoreIndex, float gradScale)
    {
        lock (_gate)
        {
            Drain();
            var l = Desc(logits);
            PaiTensor loss, grad;
            fixed (int* p = targets)
                Native.Check(Native.CrossEntropyFused(Ctx, &l, p, targets.Length, ignoreIndex, gradScale, &loss, &grad));
            return (Wrap(loss), Wrap(grad));
        }
    }

    /// <summary>One AdamW update of p, m and v in place (Optimizers.cs:81-123, same per-element operation order).</summary>
    public void AdamWStep(Tensor p, Tensor g, Tensor m, Tensor v, float lr, float beta1, float beta2, float eps,
                          float weightDecay, int t, float gradScale = 1.0f)
    {
        lock (_gate)
        {
            Drain();
            var dp = Desc(p);
            var dg = Desc(g);
            var dm = Desc(m);
            var dv = Desc(v);
            Native.Check(Native.AdamWStep(Ctx, &dp, &dg, &dm, &dv, lr, beta1, beta2, eps, weightDecay, t, gradScale));
        }
    }

    /// <summary>
    /// RMSNorm backward into caller-owned dx and dw without allocating device memory (a fixed device array holds the
    /// partial sums; calls that overlap on the GPU race on it; rows up to 8192 elements).
    /// </summary>
    public void RmsNormBackwardInto(Tensor x, Tensor weight, Tensor grad, float eps, Tensor dx, Tensor dw)
    {
        lock (_gate)
        {
            Drain();
            var a = Desc(x);
            var w = Desc(weight);
            var g = Desc(grad);
            var rx = Desc(dx);
            var rw = Desc(dw);
            Native.Check(Native.RmsNormBwdNoAlloc(Ctx, &a, &w, &g, eps, &rx, &rw));
        }
    }

    // ------------------------------------------------------------ Decode (device KV cache, graph-replayed steps)

    /// <summary>Per-row argmax of the last axis with ArgMax's rules (Sampling.cs:15-31), as float indices.</summary>
    public Tensor ArgMaxRows(Tensor x)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            PaiTensor o;
            Native.Check(Native.ArgMaxRows(Ctx, &d, &o));
            return Wrap(o);
        }
    }

    /// <summary>Host -> device copy into an existing dense tensor, ordered on the stream (decode ids and position).</summary>
    public void Write(ReadOnlySpan<float> data, Tensor destination)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(destination);
            fixed (float* p = data) Native.Check(Native.Write(Ctx, p, data.Length, &d));
        }
    }

    /// <summary>Embedding rows by ids held in a device tensor (integral float values).</summary>
    public Tensor GatherDevice(Tensor table, Tensor ids)
    {
        lock (_gate)
        {
            Drain();
            var t = Desc(table);
            var i = Desc(ids);
            PaiTensor o;
            Native.Check(Native.GatherDev(Ctx, &t, &i, &o));
            return Wrap(o);
        }
    }

    /// <summary>RoPE with the table rows chosen on the device from the position tensor.</summary>
    public Tensor RotaryAt(Tensor x, Tensor cosTable, Tensor sinTable, Tensor position)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            var c = Desc(cosTable);
            var s = Desc(sinTable);
            var p = Desc(position);
            PaiTensor o;
            Native.Check(Native.RotaryAt(Ctx, &d, &c, &s, &p, &o));
            return Wrap(o);
        }
    }

    /// <summary>Writes k and v into the preallocated caches at the device-held position (in place).</summary>
    public void KvAppend(Tensor k, Tensor v, Tensor kCache, Tensor vCache, Tensor position)
    {
        lock (_gate)
        {
            Drain();
            var dk = Desc(k);
            var dv = Desc(v);
            var kc = Desc(kCache);
            var vc = Desc(vCache);
            var p = Desc(position);
            Native.Check(Native.KvAppend(Ctx, &dk, &dv, &kc, &vc, &p));
        }
    }

    /// <summary>Decode attention over the cache prefix [0, position + rows).</summary>
    public Tensor SdpaDecode(Tensor q, Tensor kCache, Tensor vCache, Tensor position, float scale)
    {
        lock (_gate)
        {
            Drain();
            var dq = Desc(q);
            var kc = Desc(kCache);
            var vc = Desc(vCache);
            var p = Desc(position);
            PaiTensor o;
            Native.Check(Native.SdpaDecode(Ctx, &dq, &kc, &vc, &p, scale, &o));
            return Wrap(o);
        }
    }

    /// <summary>RoPE of q and k, then k and v appended to the caches; returns the rotated q.</summary>
    public Tensor RopeAppend(Tensor q, Tensor k, Tensor v, Tensor cosTable, Tensor sinTable, Tensor kCache, Tensor vCache,
                             Tensor position)
    {
        lock (_gate)
        {
            Drain();
            var dq = Desc(q);
            var dk = Desc(k);
            var dv = Desc(v);
            var c = Desc(cosTable);
            var s = Desc(sinTable);
            var kc = Desc(kCache);
            var vc = Desc(vCache);
            var p = Desc(position);
            PaiTensor o;
            Native.Check(Native.RopeAppend(Ctx, &dq, &dk, &dv, &c, &s, &kc, &vc, &p, &o));
            return Wrap(o);
        }
    }

    /// <summary>RoPE, cache append and decode attention in one launch (the values of RopeAppend + SdpaDecode).</summary>
    public Tensor AttentionDecodeStep(Tensor q, Tensor k, Tensor v, Tensor cosTable, Tensor sinTable, Tensor kCache,
                                      Tensor vCache, Tensor position, float scale)
    {
        lock (_gate)
        {
            Drain();
            var dq = Desc(q);
            var dk = Desc(k);
            var dv = Desc(v);
            var c = Desc(cosTable);
            var s = Desc(sinTable);
            var kc = Desc(kCache);
            var vc = Desc(vCache);
            var p = Desc(position);
            PaiTensor o;
            Native.Check(Native.AttnDecodeStep(Ctx, &dq, &dk, &dv, &c, &s, &kc, &vc, &p, scale, &o));
            return Wrap(o);
        }
    }

    /// <summary>
    /// Decode-step products x·W_iᵀ in one pass over the weights, optionally RMS-normalising x first: mode 0 side by
    /// side, mode 1 residual + x·W_0ᵀ, mode 2 SiLU(x·W_0ᵀ) ⊙ (x·W_1ᵀ) (include/projectai_cuda.h, pai_linear_fused).
    /// </summary>
    public Tensor LinearFused(Tensor x, Tensor? normWeight, float eps, IReadOnlyList<Tensor> weights, int mode,
                              Tensor? residual)
    {
        lock (_gate)
        {
            Drain();
            var dx = Desc(x);
            PaiTensor nw = normWeight is null ? default : Desc(normWeight);
            PaiTensor res = residual is null ? default : Desc(residual);
            var ws = new PaiTensor[weights.Count];
            for (int i = 0; i < ws.Length; i++) ws[i] = Desc(weights[i]);
            PaiTensor o;
            fixed (PaiTensor* pw = ws)
                Native.Check(Native.LinearFused(Ctx, &dx, normWeight is null ? null : &nw, eps, pw, ws.Length, mode,
                                                residual is null ? null : &res, &o));
            return Wrap(o);
        }
    }

    /// <summary>Starts capturing every op on the stream into a CUDA graph (no host sync may come before EndGraph).</summary>
    public void BeginGraph()
    {
        lock (_gate)
        {
            Drain();
            Native.Check(Native.GraphBegin(Ctx));
        }
    }

    public IntPtr EndGraph()
    {
        lock (_gate)
        {
            IntPtr g;
            Native.Check(Native.GraphEnd(Ctx, &g));
            return g;
        }
    }

    public void LaunchGraph(IntPtr graph)
    {
        lock (_gate) Native.Check(Native.GraphLaunch(Ctx, graph));
    }

    public void DestroyGraph(IntPtr graph)
    {
        lock (_gate) Native.Check(Native.GraphDestroy(Ctx, graph));
    }

    // ------------------------------------------------------------ Data parallel (one process per GPU)

    /// <summary>A new NCCL communicator id (rank 0 creates it and sends it to the other ranks).</summary>
    public static byte[] NewCommunicatorId()
    {
        var id = new byte[128];
        fixed (byte* p = id) Native.Check(Native.NcclUniqueId(p));
        return id;
    }

    /// <summary>Joins the communicator; every later call is bounded by timeoutMs (a dead peer ends in an exception).</summary>
    public void JoinDataParallel(byte[] communicatorId, int rank, int worldSize, int timeoutMs)
    {
        if (communicatorId.Length != 128) throw new ArgumentException("a communicator id is 128 bytes", nameof(communicatorId));
        lock (_gate)
        {
            Drain();
            fixed (byte* p = communicatorId) Native.Check(Native.NcclInit(Ctx, p, rank, worldSize, timeoutMs));
        }
    }

    /// <summary>
    /// The data-parallel bucket hook: sums these gradients across ranks on the communication stream, after the work
    /// queued so far (called per checkpointed block after Autograd.cs:144, and for the remaining parameters after
    /// Backward).
    /// </summary>
    public void GradientsReady(IReadOnlyList<Tensor> gradients)
    {
        lock (_gate)
        {
            Drain();
            var ds = new PaiTensor[gradients.Count];
            for (int i = 0; i < ds.Length; i++) ds[i] = Desc(gradients[i]);
            fixed (PaiTensor* p = ds) Native.Check(Native.AllreduceBucket(Ctx, p, ds.Length));
        }
    }

    /// <summary>
    /// ZeRO-1: sums these gradients across ranks leaving this rank's shard (elements [r·n/W, (r+1)·n/W) of each
    /// flattened tensor) in place, for an AdamW step on the shard alone. Every tensor's element count must divide by
    /// the world size.
    /// </summary>
    public void GradientShardsReady(IReadOnlyList<Tensor> gradients) => ShardExchange(gradients, scatter: true);

    /// <summary>ZeRO-1: copies every rank's updated shard into all ranks' parameters (after the sharded AdamW step).</summary>
    public void GatherParameterShards(IReadOnlyList<Tensor> parameters) => ShardExchange(parameters, scatter: false);

    private void ShardExchange(IReadOnlyList<Tensor> tensors, bool scatter)
    {
        lock (_gate)
        {
            Drain();
            var ds = new PaiTensor[tensors.Count];
            for (int i = 0; i < ds.Length; i++) ds[i] = Desc(tensors[i]);
            fixed (PaiTensor* p = ds)
                Native.Check(scatter ? Native.ReduceScatterBucket(Ctx, p, ds.Length) : Native.AllgatherBucket(Ctx, p, ds.Length));
        }
    }

    /// <summary>Waits (bounded) for every exchange issued so far; the optimizer step comes after.</summary>
    public void WaitForGradients()
    {
        lock (_gate) Native.Check(Native.AllreduceWait(Ctx));
    }

    public void AbortDataParallel()
    {
        lock (_gate) Native.Check(Native.NcclAbort(Ctx));
    }

    /// <summary>Exposed all-reduce device time (ms, summed) and the steps counted since the last call.</summary>
    public (double ExposedMs, long Steps) DataParallelStats()
    {
        lock (_gate)
        {
            double ms;
            long n;
            Native.Check(Native.DpStats(Ctx, &ms, &n));
            return (ms, n);
        }
    }

    // ------------------------------------------------------------ Checkpoints (ProjectAI.Formats/Checkpoint.cs)

    /// <summary>
    /// Checkpoint.Save (Checkpoint.cs:23-57) on the device's side of the copy: the tensors are snapshotted on the GPU
    /// and the PAICKPT2 file is written by a native thread while training continues; <see cref="WaitCheckpoint"/>
    /// joins it (and throws its IOException). Byte-identical to Checkpoint.Save for F32 tensors.
    /// </summary>
    public void SaveCheckpoint(string path, int step, IEnumerable<(string Name, Tensor Tensor)> tensors, string metadata = "")
    {
        var items = tensors.ToList();
        var names = new List<byte>();
        foreach (var (name, _) in items) { names.AddRange(Encoding.UTF8.GetBytes(name)); names.Add(0); }
        byte[] nameBytes = names.ToArray(), pathBytes = Encoding.UTF8.GetBytes(path + "\0"), meta = Encoding.UTF8.GetBytes(metadata);
        lock (_gate)
        {
            Drain();
            var ds = new PaiTensor[Math.Max(1, items.Count)];
            for (int i = 0; i < items.Count; i++) ds[i] = Desc(items[i].Tensor);
            fixed (byte* pp = pathBytes) fixed (byte* pm = meta) fixed (byte* pn = nameBytes) fixed (PaiTensor* pt = ds)
                Native.Check(Native.CkptSave(Ctx, pp, step, pm, meta.Length, pn, nameBytes.Length, pt, items.Count));
        }
    }

    public void WaitCheckpoint()
    {
        lock (_gate) Native.Check(Native.CkptWait(Ctx));
    }

    /// <summary>Checkpoint.Load (Checkpoint.cs:59-110): step, metadata and the tensors by name, on this device.</summary>
    public (int Step, string Metadata, IReadOnlyList<(string Name, Tensor Tensor)> Tensors) LoadCheckpoint(string path)
    {
        var (step, meta, count) = ReadCheckpointHeader(path, headerOnly: false);
        var list = new List<(string, Tensor)>(count);
        lock (_gate)
        {
            for (int i = 0; i < count; i++)
            {
                long len;
                Native.Check(Native.CkptTensor(Ctx, i, null, 0, &len, null));
                var name = new byte[Math.Max(1, len)];
                PaiTensor d;
                fixed (byte* pn = name) Native.Check(Native.CkptTensor(Ctx, i, pn, len, null, &d));
                list.Add((Encoding.UTF8.GetString(name, 0, (int)len), Wrap(d)));
            }
            Native.Check(Native.CkptClose(Ctx));
        }
        return (step, meta, list);
    }

    /// <summary>Checkpoint.ReadMetadata (Checkpoint.cs:113-129): the step and metadata from the header alone.</summary>
    public (int Step, string Metadata) ReadCheckpointMetadata(string path)
    {
        var (step, meta, _) = ReadCheckpointHeader(path, headerOnly: true);
        lock (_gate) Native.Check(Native.CkptClose(Ctx));
        return (step, meta);
    }

    private (int Step, string Metadata, int Count) ReadCheckpointHeader(string path, bool headerOnly)
    {
        byte[] pathBytes = Encoding.UTF8.GetBytes(path + "\0");
        lock (_gate)
        {
            Drain();
            int step, count;
            long metaLen;
            fixed (byte* pp = pathBytes) Native.Check(Native.CkptLoad(Ctx, pp, headerOnly ? 1 : 0, &step, &metaLen, &count));
            var meta = new byte[Math.Max(1, metaLen)];
            fixed (byte* pm = meta) Native.Check(Native.CkptMeta(Ctx, pm, metaLen));
            return (step, Encoding.UTF8.GetString(meta, 0, (int)metaLen), count);
        }
    }

    // ------------------------------------------------------------ Packed datasets (ProjectAI.Training/PackedBinDataset.cs)

    /// <summary>
    /// Maps the shard a packed dataset's manifest names (PackedBinDataset.Open, PackedBinDataset.cs:43-95, after the
    /// manifest is read): dtype "u16" or "u32", blocks of sequenceLength + 1 ids.
    /// </summary>
    public void OpenDataset(string shardPath, string dtype, int sequenceLength, long blockCount)
    {
        byte[] pathBytes = Encoding.UTF8.GetBytes(shardPath + "\0");
        int width = dtype switch { "u16" => 2, "u32" => 4, _ => 0 };
        lock (_gate)
            fixed (byte* pp = pathBytes) Native.Check(Native.DatasetOpen(Ctx, pp, width, sequenceLength, blockCount));
    }

    /// <summary>
    /// Trainer.NextBatch (Training.cs:122-141) for the given block indices, ids straight to the device: the blocks are
    /// gathered from the mapped shard, uploaded at their on-disk width and widened to the F32 input and target ids on
    /// the GPU.
    /// </summary>
    public (Tensor Input, Tensor Target) NextBatch(IReadOnlyList<long> blockIndices)
    {
        var idx = blockIndices.ToArray();
        lock (_gate)
        {
            Drain();
            PaiTensor i, t;
            fixed (long* p = idx) Native.Check(Native.DatasetBatch(Ctx, p, idx.Length, &i, &t));
            return (Wrap(i), Wrap(t));
        }
    }

    public void CloseDataset()
    {
        lock (_gate) Native.Check(Native.DatasetClose(Ctx));
    }

    // ------------------------------------------------------------ Diagnostics

    public void Synchronize()
    {
        lock (_gate) Native.Check(Native.Sync(Ctx));
    }

    public (long InUse, long Peak, long Reserved) MemoryStats()
    {
        lock (_gate)
        {
            long a, b, c;
            Native.Check(Native.MemoryStats(Ctx, &a, &b, &c));
            return (a, b, c);
        }
    }

    public void ResetPeakMemory()
    {
        lock (_gate) Native.Check(Native.ResetPeak(Ctx));
    }

    /// <summary>Throws if a kernel's bounded wait timed out since the last check (the launch's results are invalid).</summary>
    public void CheckDeviceError()
    {
        lock (_gate)
        {
            int code;
            Native.Check(Native.CheckDeviceError(Ctx, &code));
        }
    }

    public void StartTimer()
    {
        lock (_gate) Native.Check(Native.TimerStart(Ctx));
    }

    /// <summary>Device milliseconds since StartTimer, from CUDA events on the stream (waits for the stream).</summary>
    public float StopTimer()
    {
        lock (_gate)
        {
            float ms;
            Native.Check(Native.TimerStop(Ctx, &ms));
            return ms;
        }
    }

    public long LaunchCount()
    {
        lock (_gate)
        {
            long n;
            Native.Check(Native.LaunchCount(Ctx, &n));
            return n;
        }
    }

    public void KernelTiming(bool enable)
    {
        lock (_gate) Native.Check(Native.KernelTiming(Ctx, enable ? 1 : 0));
    }

    /// <summary>Launches, summed device ms and summed algorithmic work of a kernel family ("gemm", "attn_fwd", ...).</summary>
    public (long Launches, double TotalMs, double Work) KernelStats(string family)
    {
        byte[] name = Encoding.UTF8.GetBytes(family + "\0");
        lock (_gate)
        {
            long n;
            double ms, work;
            fixed (byte* p = name) Native.Check(Native.KernelStats(Ctx, p, &n, &ms, &work));
            return (n, ms, work);
        }
    }

    // ------------------------------------------------------------ plumbing

    private IntPtr Ctx => _ctx != IntPtr.Zero ? _ctx : throw new ObjectDisposedException(nameof(CudaComputeBackend));

    internal void EnqueueFinalized(CudaBuffer buffer) => _finalized.Enqueue(buffer);

    // Frees the blocks whose last view the GC collected since the previous call, on the caller's thread (the GC path,
    // pai_finalize). A block an open scope owns is left to that scope, which frees it when it ends.
    private void Drain()
    {
        while (_finalized.TryDequeue(out var b))
        {
            if (b.Freed || _ctx == IntPtr.Zero || b.Scope >= 0) continue;
            b.Freed = true;
            Native.Check(Native.Finalize(Ctx, b.Base));
        }
    }

    private void Free(CudaBuffer b)
    {
        b.Freed = true;
        if (b.Scope >= 0 && b.Scope < _scopes.Count) _scopes[b.Scope].Remove(b);
        Native.Check(Native.Release(Ctx, b.Base));
    }

    private CudaBuffer Buffer(Tensor t)
    {
        if (t.Handle is not CudaBuffer b || !ReferenceEquals(b.Owner, this))
            throw new ArgumentException("the tensor was not created by this CUDA backend");
        return b;
    }

    private PaiTensor Desc(Tensor t)
    {
        var b = Buffer(t);
        if (b.Freed) throw new InvalidOperationException("the tensor's memory was released (scope ended or Release)");
        var dims = t.Shape.Dimensions;
        if (dims.Length > PaiTensor.MaxRank) throw new ArgumentException($"rank {dims.Length} above {PaiTensor.MaxRank}");
        var d = new PaiTensor { Base = b.Base, Offset = t.Offset, Rank = dims.Length, DType = (int)t.DType };
        for (int i = 0; i < dims.Length; i++)
        {
            d.Dims[i] = dims[i];
            d.Strides[i] = t.Strides[i];
        }
        return d;
    }

    private Tensor Wrap(PaiTensor d)
    {
        var dims = new int[d.Rank];
        for (int i = 0; i < d.Rank; i++) dims[i] = d.Dims[i];
        var b = new CudaBuffer(this, d.Base, _scopes.Count - 1);
        if (_scopes.Count > 0) _scopes[^1].Add(b);
        return new Tensor(new Shape(dims), (DType)d.DType, Device, handle: b);
    }

    private static int Dims(Shape shape, int* dims)
    {
        var s = shape.Dimensions;
        if (s.Length > PaiTensor.MaxRank) throw new ArgumentException($"rank {s.Length} above {PaiTensor.MaxRank}");
        for (int i = 0; i < s.Length; i++) dims[i] = s[i];
        return s.Length;
    }

    private static int IndexOfZero(byte* p, int n)
    {
        for (int i = 0; i < n; i++)
            if (p[i] == 0) return i;
        return n;
    }

    private Tensor Binary(Tensor a, Tensor b, int op)
    {
        lock (_gate)
        {
            Drain();
            var x = Desc(a);
            var y = Desc(b);
            PaiTensor o;
            int st = op switch
            {
                0 => Native.Add(Ctx, &x, &y, &o),
                1 => Native.Mul(Ctx, &x, &y, &o),
                2 => Native.Sub(Ctx, &x, &y, &o),
                _ => Native.Div(Ctx, &x, &y, &o),
            };
            Native.Check(st);
            return Wrap(o);
        }
    }

    private Tensor Unary(Tensor x, int op)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            PaiTensor o;
            int st = op switch
            {
                0 => Native.Sqrt(Ctx, &d, &o),
                1 => Native.Sigmoid(Ctx, &d, &o),
                _ => Native.Silu(Ctx, &d, &o),
            };
            Native.Check(st);
            return Wrap(o);
        }
    }

    private Tensor Reduce(Tensor x, int axis, bool keepDims, int op)
    {
        lock (_gate)
        {
            Drain();
            var d = Desc(x);
            PaiTensor o;
            int keep = keepDims ? 1 : 0;
            int st = op switch
            {
                0 => Native.Sum(Ctx, &d, axis, keep, &o),
                1 => Native.Mean(Ctx, &d, axis, keep, &o),
                _ => Native.Max(Ctx, &d, axis, keep, &o),
            };
            Native.Check(st);
            return Wrap(o);
        }
    }
}
