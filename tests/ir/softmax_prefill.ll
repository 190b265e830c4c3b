; softmax_prefill.ll -- causal paged prefill attention over query tiles, fp32.
; Grid (tiles, Hq): ctaid.x = query tile (the task axis pi remaps), ctaid.y =
; query head h (KV head h / G); thread tid.x = row r of the tile (<= 16 rows).
; tiles[x] = (req, q_row0, nq, q_pos0) as int32; the row at absolute position
; p = q_pos0 + r attends to the request's keys [0, p] through its block table.
;   q, out [row][Hq][64]    kc, vc [page][Hkv][16][64]    bt [req][maxp]
; Online softmax per row (llvm.maxnum + llvm.exp2 in the log2 domain), as the
; decode fixture; the key loop's IV %t is the canonical IV.
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.y()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()
declare float @llvm.maxnum.f32(float, float)
declare float @llvm.exp2.f32(float)

define ptx_kernel void @softmax_prefill(ptr %q, ptr %kc, ptr %vc, ptr %bt, ptr %tiles, ptr %out, ptr %acc, i32 %maxp, i32 %G, i32 %Hq, float %scale) {
entry:
  %tile = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %h = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.y()
  %r = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %tp = mul i32 %tile, 4
  %req.gep = getelementptr i32, ptr %tiles, i32 %tp
  %req = load i32, ptr %req.gep, align 4
  %tp1 = add i32 %tp, 1
  %row0.gep = getelementptr i32, ptr %tiles, i32 %tp1
  %row0 = load i32, ptr %row0.gep, align 4
  %tp2 = add i32 %tp, 2
  %nq.gep = getelementptr i32, ptr %tiles, i32 %tp2
  %nq = load i32, ptr %nq.gep, align 4
  %tp3 = add i32 %tp, 3
  %pos0.gep = getelementptr i32, ptr %tiles, i32 %tp3
  %pos0 = load i32, ptr %pos0.gep, align 4
  %live = icmp slt i32 %r, %nq
  br i1 %live, label %go, label %ret

go:
  %row = add i32 %row0, %r
  %qpos = add i32 %pos0, %r
  %n = add i32 %qpos, 1
  %rh0 = mul i32 %row, %Hq
  %rh = add i32 %rh0, %h
  %qbase = mul i32 %rh, 64
  %hkv = udiv i32 %h, %G
  %Hkv = udiv i32 %Hq, %G
  %btrow = mul i32 %req, %maxp
  br label %zero

zero:
  %z = phi i32 [ 0, %go ], [ %z.next, %zero ]
  %zi = add i32 %qbase, %z
  %z.gep = getelementptr float, ptr %acc, i32 %zi
  store float 0.000000e+00, ptr %z.gep, align 4
  %z.next = add i32 %z, 1
  %z.done = icmp eq i32 %z.next, 64
  br i1 %z.done, label %tok, label %zero

tok:
  %t = phi i32 [ 0, %zero ], [ %t.next, %tok.latch ]
  %m = phi float [ 0xFFF0000000000000, %zero ], [ %m.next, %tok.latch ]
  %l = phi float [ 0.000000e+00, %zero ], [ %l.next, %tok.latch ]
  %pidx = lshr i32 %t, 4
  %slot = and i32 %t, 15
  %bt.i = add i32 %btrow, %pidx
  %bt.gep = getelementptr i32, ptr %bt, i32 %bt.i
  %page = load i32, ptr %bt.gep, align 4
  %ph = mul i32 %page, %Hkv
  %ph2 = add i32 %ph, %hkv
  %p16 = mul i32 %ph2, 16
  %kvrow = add i32 %p16, %slot
  %kvbase = mul i32 %kvrow, 64
  br label %dot

dot:
  %d = phi i32 [ 0, %tok ], [ %d.next, %dot ]
  %s.acc = phi float [ 0.000000e+00, %tok ], [ %s.next, %dot ]
  %qi = add i32 %qbase, %d
  %q.gep = getelementptr float, ptr %q, i32 %qi
  %qv = load float, ptr %q.gep, align 4
  %ki = add i32 %kvbase, %d
  %k.gep = getelementptr float, ptr %kc, i32 %ki
  %kv = load float, ptr %k.gep, align 4
  %s.next = call float @llvm.fma.f32(float %qv, float %kv, float %s.acc)
  %d.next = add i32 %d, 1
  %d.done = icmp eq i32 %d.next, 64
  br i1 %d.done, label %upd, label %dot

upd:
  %s = fmul float %s.next, %scale
  %m.next = call float @llvm.maxnum.f32(float %m, float %s)
  %dm = fsub float %m, %m.next
  %alpha = call float @llvm.exp2.f32(float %dm)
  %ds = fsub float %s, %m.next
  %p = call float @llvm.exp2.f32(float %ds)
  %la = fmul float %l, %alpha
  %l.next = fadd float %la, %p
  br label %pv

pv:
  %e = phi i32 [ 0, %upd ], [ %e.next, %pv ]
  %ai = add i32 %qbase, %e
  %a.gep = getelementptr float, ptr %acc, i32 %ai
  %av = load float, ptr %a.gep, align 4
  %vi = add i32 %kvbase, %e
  %v.gep = getelementptr float, ptr %vc, i32 %vi
  %vv = load float, ptr %v.gep, align 4
  %pvv = fmul float %p, %vv
  %as = fmul float %av, %alpha
  %an = fadd float %as, %pvv
  store float %an, ptr %a.gep, align 4
  %e.next = add i32 %e, 1
  %e.done = icmp eq i32 %e.next, 64
  br i1 %e.done, label %tok.latch, label %pv

tok.latch:
  %t.next = add i32 %t, 1
  %t.done = icmp eq i32 %t.next, %n
  br i1 %t.done, label %fin, label %tok

fin:
  %inv = fdiv float 1.000000e+00, %l.next
  br label %wr

wr:
  %o = phi i32 [ 0, %fin ], [ %o.next, %wr ]
  %oi = add i32 %qbase, %o
  %oa.gep = getelementptr float, ptr %acc, i32 %oi
  %oa = load float, ptr %oa.gep, align 4
  %ov = fmul float %oa, %inv
  %oo.gep = getelementptr float, ptr %out, i32 %oi
  store float %ov, ptr %oo.gep, align 4
  %o.next = add i32 %o, 1
  %o.done = icmp eq i32 %o.next, 64
  br i1 %o.done, label %ret, label %wr

ret:
  ret void
}

declare float @llvm.fma.f32(float, float, float)
