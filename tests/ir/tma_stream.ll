; tma_stream.ll -- a contraction whose stream arrives by TMA (the pattern of
; tcgen05 producers): per iteration k, thread 0 arms the stage barrier and
; loads the 64 x 8 bf16 box at coordinates {k * 64, req * 8} of a 2-D tensor
; map into shared memory; every thread then polls the barrier once and reads
; one element. The box's innermost coordinate is affine in the canonical IV
; %k (step 64); the row coordinate is loop-invariant. Woven and assembled
; for sm_100a only (it is never executed).
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8
@smem = internal addrspace(3) global [512 x i16] undef, align 128
@bar = internal addrspace(3) global i64 undef, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()

define ptx_kernel void @tma_stream(ptr %tmap, ptr %out, i32 %n) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %t = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %y = mul i32 %req, 8
  %dst = ptrtoint ptr addrspace(3) @smem to i32
  %mb = ptrtoint ptr addrspace(3) @bar to i32
  %lead = icmp eq i32 %t, 0
  %leadi = zext i1 %lead to i32
  %sh = getelementptr [512 x i16], ptr addrspace(3) @smem, i32 0, i32 %t
  br label %loop

loop:
  %k = phi i32 [ 0, %entry ], [ %k.next, %loop ]
  %acc = phi i32 [ 0, %entry ], [ %acc.next, %loop ]
  %x = mul i32 %k, 64
  %ph = and i32 %k, 1
  call void asm sideeffect "{ .reg .pred p; setp.ne.u32 p, $5, 0; @p mbarrier.arrive.expect_tx.shared::cta.b64 _, [$4], 1024; @p cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [$0], [$1, {$2, $3}], [$4]; }", "r,l,r,r,r,r,~{memory}"(i32 %dst, ptr %tmap, i32 %x, i32 %y, i32 %mb, i32 %leadi)
  call void asm sideeffect "{ .reg .pred q; mbarrier.try_wait.parity.shared::cta.b64 q, [$0], $1; }", "r,r,~{memory}"(i32 %mb, i32 %ph)
  %v = load i16, ptr addrspace(3) %sh, align 2
  %vz = zext i16 %v to i32
  %acc.next = add i32 %acc, %vz
  %k.next = add i32 %k, 1
  %done = icmp eq i32 %k.next, %n
  br i1 %done, label %exit, label %loop

exit:
  %o0 = mul i32 %req, 128
  %o = add i32 %o0, %t
  %og = getelementptr i32, ptr %out, i32 %o
  store i32 %acc.next, ptr %og, align 4
  ret void
}
