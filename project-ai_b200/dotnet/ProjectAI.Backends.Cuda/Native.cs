// P/Invoke bindings of libprojectai_cuda.so: one LibraryImport per entry point of include/projectai_cuda.h, with the
// same argument order and meaning. Every import returns the C status (0 = success) except LastError; Check turns a
// status into the exception the reference throws for the same condition (the header's "Conventions" block).
//
// Type mapping: pai_ctx* / pai_graph* / a block base (const void*) -> IntPtr; const pai_tensor* / pai_tensor* ->
// PaiTensor*; const float* / float* -> float*; const int32_t* -> int*; int64_t* -> long*; uint8_t[128] and char* ->
// byte*; int32_t -> int; int64_t -> long.
using System.Runtime.InteropServices;

namespace ProjectAI.Backends.Cuda;

/// <summary>include/projectai_cuda.h: pai_tensor (a view: storage base, element offset, shape, element strides).</summary>
[StructLayout(LayoutKind.Sequential)]
internal unsafe struct PaiTensor
{
    public const int MaxRank = 8;
    public IntPtr Base;
    public long Offset;
    public int Rank;
    public int DType;
    public fixed int Dims[MaxRank];
    public fixed long Strides[MaxRank];
}

/// <summary>include/projectai_cuda.h: pai_status.</summary>
internal enum PaiStatus
{
    Ok = 0,
    Argument = 1,
    OutOfRange = 2,
    InvalidOperation = 3,
    OutOfMemory = 4,
    Cuda = 5,
    Nccl = 6,
    Timeout = 7,
    Unsupported = 8,
    Io = 9,
    InvalidData = 10,
}

internal static unsafe partial class Native
{
    private const string Lib = "projectai_cuda";

    [LibraryImport(Lib, EntryPoint = "pai_last_error")] internal static partial IntPtr LastError();
    [LibraryImport(Lib, EntryPoint = "pai_ctx_create")] internal static partial int CtxCreate(int deviceOrdinal, IntPtr* @out);
    [LibraryImport(Lib, EntryPoint = "pai_ctx_destroy")] internal static partial int CtxDestroy(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_sync")] internal static partial int Sync(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_device_name")] internal static partial int DeviceName(IntPtr ctx, byte* buf, int bufLen);
    [LibraryImport(Lib, EntryPoint = "pai_alloc")] internal static partial int Alloc(IntPtr ctx, int rank, int* dims, int dtype, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_from_host")] internal static partial int FromHost(IntPtr ctx, float* host, long count, int rank, int* dims, int dtype, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_to_host")] internal static partial int ToHost(IntPtr ctx, PaiTensor* src, float* host, long count);
    [LibraryImport(Lib, EntryPoint = "pai_copy")] internal static partial int Copy(IntPtr ctx, PaiTensor* src, PaiTensor* dst);
    [LibraryImport(Lib, EntryPoint = "pai_scope_begin")] internal static partial int ScopeBegin(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_scope_end")] internal static partial int ScopeEnd(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_keep_alive")] internal static partial int KeepAlive(IntPtr ctx, IntPtr @base);
    [LibraryImport(Lib, EntryPoint = "pai_release")] internal static partial int Release(IntPtr ctx, IntPtr @base);
    [LibraryImport(Lib, EntryPoint = "pai_finalize")] internal static partial int Finalize(IntPtr ctx, IntPtr @base);
    [LibraryImport(Lib, EntryPoint = "pai_memory_stats")] internal static partial int MemoryStats(IntPtr ctx, long* inUse, long* peak, long* reserved);
    [LibraryImport(Lib, EntryPoint = "pai_reset_peak")] internal static partial int ResetPeak(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_add")] internal static partial int Add(IntPtr ctx, PaiTensor* a, PaiTensor* b, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sub")] internal static partial int Sub(IntPtr ctx, PaiTensor* a, PaiTensor* b, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_mul")] internal static partial int Mul(IntPtr ctx, PaiTensor* a, PaiTensor* b, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_div")] internal static partial int Div(IntPtr ctx, PaiTensor* a, PaiTensor* b, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_add_scalar")] internal static partial int AddScalar(IntPtr ctx, PaiTensor* a, float scalar, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_mul_scalar")] internal static partial int MulScalar(IntPtr ctx, PaiTensor* a, float scalar, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sqrt")] internal static partial int Sqrt(IntPtr ctx, PaiTensor* x, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sigmoid")] internal static partial int Sigmoid(IntPtr ctx, PaiTensor* x, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_matmul")] internal static partial int MatMul(IntPtr ctx, PaiTensor* a, PaiTensor* b, int transposeB, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sum")] internal static partial int Sum(IntPtr ctx, PaiTensor* x, int axis, int keepDims, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_mean")] internal static partial int Mean(IntPtr ctx, PaiTensor* x, int axis, int keepDims, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_max")] internal static partial int Max(IntPtr ctx, PaiTensor* x, int axis, int keepDims, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_argmax_rows")] internal static partial int ArgMaxRows(IntPtr ctx, PaiTensor* x, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_softmax")] internal static partial int Softmax(IntPtr ctx, PaiTensor* x, int axis, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_rmsnorm")] internal static partial int RmsNorm(IntPtr ctx, PaiTensor* x, PaiTensor* weight, float eps, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_silu")] internal static partial int Silu(IntPtr ctx, PaiTensor* x, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_rotary")] internal static partial int Rotary(IntPtr ctx, PaiTensor* x, PaiTensor* cos, PaiTensor* sin, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_gather")] internal static partial int Gather(IntPtr ctx, PaiTensor* table, int* ids, long nIds, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_scatter_add_rows")] internal static partial int ScatterAddRows(IntPtr ctx, PaiTensor* rows, int* ids, long nIds, int rowCount, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_cross_entropy")] internal static partial int CrossEntropy(IntPtr ctx, PaiTensor* logits, int* targets, long nTargets, int ignoreIndex, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_cross_entropy_grad")] internal static partial int CrossEntropyGrad(IntPtr ctx, PaiTensor* logits, int* targets, long nTargets, int ignoreIndex, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_cat")] internal static partial int Cat(IntPtr ctx, PaiTensor* a, PaiTensor* b, int axis, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sdpa_fwd")] internal static partial int SdpaFwd(IntPtr ctx, PaiTensor* q, PaiTensor* k, PaiTensor* v, float scale, int causal, int posOffset, PaiTensor* @out, PaiTensor* lse);
    [LibraryImport(Lib, EntryPoint = "pai_sdpa_bwd")] internal static partial int SdpaBwd(IntPtr ctx, PaiTensor* q, PaiTensor* k, PaiTensor* v, PaiTensor* @out, PaiTensor* lse, PaiTensor* dout, float scale, int causal, int posOffset, PaiTensor* dq, PaiTensor* dk, PaiTensor* dv);
    [LibraryImport(Lib, EntryPoint = "pai_rmsnorm_bwd")] internal static partial int RmsNormBwd(IntPtr ctx, PaiTensor* x, PaiTensor* weight, PaiTensor* g, float eps, PaiTensor* dx, PaiTensor* dw);
    [LibraryImport(Lib, EntryPoint = "pai_silu_mul_fwd")] internal static partial int SiluMulFwd(IntPtr ctx, PaiTensor* gate, PaiTensor* up, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_silu_mul_bwd")] internal static partial int SiluMulBwd(IntPtr ctx, PaiTensor* gate, PaiTensor* up, PaiTensor* g, PaiTensor* dgate, PaiTensor* dup);
    [LibraryImport(Lib, EntryPoint = "pai_cross_entropy_fused")] internal static partial int CrossEntropyFused(IntPtr ctx, PaiTensor* logits, int* targets, long nTargets, int ignoreIndex, float gradScale, PaiTensor* loss, PaiTensor* grad);
    [LibraryImport(Lib, EntryPoint = "pai_adamw_step")] internal static partial int AdamWStep(IntPtr ctx, PaiTensor* p, PaiTensor* g, PaiTensor* m, PaiTensor* v, float lr, float beta1, float beta2, float eps, float weightDecay, int t, float gradScale);
    [LibraryImport(Lib, EntryPoint = "pai_rmsnorm_bwd_noalloc")] internal static partial int RmsNormBwdNoAlloc(IntPtr ctx, PaiTensor* x, PaiTensor* weight, PaiTensor* g, float eps, PaiTensor* dx, PaiTensor* dw);
    [LibraryImport(Lib, EntryPoint = "pai_write")] internal static partial int Write(IntPtr ctx, float* host, long count, PaiTensor* dst);
    [LibraryImport(Lib, EntryPoint = "pai_gather_dev")] internal static partial int GatherDev(IntPtr ctx, PaiTensor* table, PaiTensor* ids, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_rotary_at")] internal static partial int RotaryAt(IntPtr ctx, PaiTensor* x, PaiTensor* cosTable, PaiTensor* sinTable, PaiTensor* pos, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_kv_append")] internal static partial int KvAppend(IntPtr ctx, PaiTensor* k, PaiTensor* v, PaiTensor* kCache, PaiTensor* vCache, PaiTensor* pos);
    [LibraryImport(Lib, EntryPoint = "pai_rope_append")] internal static partial int RopeAppend(IntPtr ctx, PaiTensor* q, PaiTensor* k, PaiTensor* v, PaiTensor* cosTable, PaiTensor* sinTable, PaiTensor* kCache, PaiTensor* vCache, PaiTensor* pos, PaiTensor* qOut);
    [LibraryImport(Lib, EntryPoint = "pai_attn_decode_step")] internal static partial int AttnDecodeStep(IntPtr ctx, PaiTensor* q, PaiTensor* k, PaiTensor* v, PaiTensor* cosTable, PaiTensor* sinTable, PaiTensor* kCache, PaiTensor* vCache, PaiTensor* pos, float scale, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_sdpa_decode")] internal static partial int SdpaDecode(IntPtr ctx, PaiTensor* q, PaiTensor* kCache, PaiTensor* vCache, PaiTensor* pos, float scale, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_linear_fused")] internal static partial int LinearFused(IntPtr ctx, PaiTensor* x, PaiTensor* normWeight, float eps, PaiTensor* weights, int nWeights, int mode, PaiTensor* residual, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_graph_begin")] internal static partial int GraphBegin(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_graph_end")] internal static partial int GraphEnd(IntPtr ctx, IntPtr* graph);
    [LibraryImport(Lib, EntryPoint = "pai_graph_launch")] internal static partial int GraphLaunch(IntPtr ctx, IntPtr graph);
    [LibraryImport(Lib, EntryPoint = "pai_graph_destroy")] internal static partial int GraphDestroy(IntPtr ctx, IntPtr graph);
    [LibraryImport(Lib, EntryPoint = "pai_nccl_unique_id")] internal static partial int NcclUniqueId(byte* idOut);
    [LibraryImport(Lib, EntryPoint = "pai_nccl_init")] internal static partial int NcclInit(IntPtr ctx, byte* id, int rank, int worldSize, int timeoutMs);
    [LibraryImport(Lib, EntryPoint = "pai_allreduce_bucket")] internal static partial int AllreduceBucket(IntPtr ctx, PaiTensor* tensors, int nTensors);
    [LibraryImport(Lib, EntryPoint = "pai_reduce_scatter_bucket")] internal static partial int ReduceScatterBucket(IntPtr ctx, PaiTensor* tensors, int nTensors);
    [LibraryImport(Lib, EntryPoint = "pai_allgather_bucket")] internal static partial int AllgatherBucket(IntPtr ctx, PaiTensor* tensors, int nTensors);
    [LibraryImport(Lib, EntryPoint = "pai_allreduce_wait")] internal static partial int AllreduceWait(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_nccl_abort")] internal static partial int NcclAbort(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_dp_stats")] internal static partial int DpStats(IntPtr ctx, double* exposedMs, long* steps);
    [LibraryImport(Lib, EntryPoint = "pai_check_device_error")] internal static partial int CheckDeviceError(IntPtr ctx, int* code);
    [LibraryImport(Lib, EntryPoint = "pai_timer_start")] internal static partial int TimerStart(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_timer_stop")] internal static partial int TimerStop(IntPtr ctx, float* ms);
    [LibraryImport(Lib, EntryPoint = "pai_launch_count")] internal static partial int LaunchCount(IntPtr ctx, long* n);
    [LibraryImport(Lib, EntryPoint = "pai_kernel_timing")] internal static partial int KernelTiming(IntPtr ctx, int enable);
    [LibraryImport(Lib, EntryPoint = "pai_kernel_stats")] internal static partial int KernelStats(IntPtr ctx, byte* family, long* launches, double* totalMs, double* work);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_save")] internal static partial int CkptSave(IntPtr ctx, byte* path, int step, byte* metadata, long metaLen, byte* names, long namesLen, PaiTensor* tensors, int nTensors);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_wait")] internal static partial int CkptWait(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_load")] internal static partial int CkptLoad(IntPtr ctx, byte* path, int headerOnly, int* step, long* metaLen, int* nTensors);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_meta")] internal static partial int CkptMeta(IntPtr ctx, byte* buf, long cap);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_tensor")] internal static partial int CkptTensor(IntPtr ctx, int index, byte* name, long nameCap, long* nameLen, PaiTensor* @out);
    [LibraryImport(Lib, EntryPoint = "pai_ckpt_close")] internal static partial int CkptClose(IntPtr ctx);
    [LibraryImport(Lib, EntryPoint = "pai_dataset_open")] internal static partial int DatasetOpen(IntPtr ctx, byte* binPath, int elemBytes, int seqLen, long blockCount);
    [LibraryImport(Lib, EntryPoint = "pai_dataset_batch")] internal static partial int DatasetBatch(IntPtr ctx, long* indices, int count, PaiTensor* inputs, PaiTensor* targets);
    [LibraryImport(Lib, EntryPoint = "pai_dataset_close")] internal static partial int DatasetClose(IntPtr ctx);


    /// <summary>The message pai_last_error() holds for this thread.</summary>
    internal static string LastMessage() => Marshal.PtrToStringUTF8(LastError()) ?? "";

    /// <summary>
    /// Maps a status onto the exception ProjectAI's CPU backend throws for the same condition: ArgumentException
    /// (shape, rank, broadcast), ArgumentOutOfRangeException (axis, id, target; CpuComputeBackend.cs:257-258,432,446,
    /// 463), InvalidOperationException, and OutOfMemoryException whose message contains "out of memory"
    /// (ProjectAI.Trainer/Program.cs:152-157 matches on that text), and for the checkpoint and dataset files the
    /// IOException and InvalidDataException of ProjectAI.Formats/Checkpoint.cs and PackedBinDataset.cs. Device, NCCL
    /// and timeout failures are InvalidOperationException with the library's message.
    /// </summary>
    internal static void Check(int status)
    {
        if (status == (int)PaiStatus.Ok) return;
        string msg = LastMessage();
        throw (PaiStatus)status switch
        {
            PaiStatus.Argument => new ArgumentException(msg),
            PaiStatus.OutOfRange => new ArgumentOutOfRangeException(null, msg),
            PaiStatus.OutOfMemory => new OutOfMemoryException(msg),
            PaiStatus.Unsupported => new NotSupportedException(msg),
            PaiStatus.Io => new IOException(msg),
            PaiStatus.InvalidData => new InvalidDataException(msg),
            _ => new InvalidOperationException(msg),
        };
    }
}
