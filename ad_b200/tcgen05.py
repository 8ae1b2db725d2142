"""Dot products on the 5th-generation tensor cores (tcgen05 + TMEM), 3xTF32.

Reference semantics: ``C[ty,tx] = sum_k A(_x=ty,_y=k) * B(_x=k,_y=tx)`` in fp32
(autodiff/device/opencl/kernels/dotprod.py:7-43) with the fused epilogue of
dp_elw_fuse.py:11-65.  B200 schedule for one dot command, or for a group of
dot commands whose kernels differ only in their buffers (``GroupPlan``):

1. ``split`` (one launch): gather every distinct A and B operand through its
   access expression (any folded Permute/View/Broadcast/Concat, or a
   constant) and write it K-major, zero-padded to the tile grid, as two fp32
   arrays ``hi = tf32_rn(x)`` and ``lo = tf32_rn(x - hi)``; operands of a
   group are stacked, operands shared by several members are split once.
2. ``gemm``: a persistent, warp-specialised kernel over all work units (tile x
   K slice x member).  Warp 0 lane 0 issues TMA loads (16 fp32 of K per row,
   SWIZZLE_64B) of A_hi, A_lo, B_hi, B_lo into a 4-stage ring; warp 1 lane 0
   issues, per 8-deep K slice, ``A_hi*B_hi + A_hi*B_lo + A_lo*B_hi`` as three
   ``tcgen05.mma.kind::tf32`` into a TMEM accumulator (the published 3xTF32
   split; the dropped ``lo*lo`` term is below fp32 rounding), with two
   accumulators so the epilogue of one tile overlaps the next tile's MMAs;
   warps 2-9 read TMEM (``tcgen05.ld.32x32b.x32``), transpose 32x32 blocks
   through shared memory for coalesced stores, and run the fused epilogue.
   Members sharing A with narrow B run as N-fused segments (one wide
   product per shared A).
3. ``splitk_epilogue`` (only when K is split or the epilogue is estimated
   faster on its own): sums the K slices in order and runs the epilogue.

Every mbarrier wait is bounded; on timeout the kernel records an error code
in a device flag, stops issuing work, drains its copies, frees its TMEM and
returns.  No TMA multicast is used anywhere.
"""
from __future__ import annotations

import ctypes
import re
from typing import Dict, List

from . import codegen, exprs, ir
from .codegen import Emitter, KernelSpec, cmd_buffers, dot_epilogue, dot_shape, index_type

import os

BM = 128
BK = 32                 # K padding of the split operands (multiple of every stage depth)
BN_DEFAULT = 256
# fp32 of K per stage row: 16 (64-byte rows, SWIZZLE_64B) or 32 (128-byte rows, SWIZZLE_128B)
BKF = int(os.environ.get("AD_GEMM_BK", "16"))
GROUP_M = int(os.environ.get("AD_GEMM_GROUP", "16"))
# K blocks accumulated in TMEM before the epilogue warps add them into fp32 running
# sums (0: the whole K slice in one TMEM accumulator).  The tensor core's fp32
# accumulation truncates (a bias toward zero of ~0.4 ulp per MMA accumulate), so
# the error of a product grows with the K it accumulates in one place.
# Off by default: measured on the config-4 step it costs 29% (4.74 vs 3.67 ms at 4 K blocks).


def fold_kb() -> int:
    return int(os.environ.get("AD_GEMM_FOLD", "0"))
SMEM_STAGES_BYTES = 192 * 1024


def stages_for(bn: int, bkf: int = BKF) -> int:
    return max(2, SMEM_STAGES_BYTES // (2 * (128 + bn) * bkf * 4))


def pad(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def tile_n(N: int) -> int:
    return 256 if N > 128 else (128 if N > 64 else 64)


# ---------------------------------------------------------------- split kernel

_SPLIT_CACHE: Dict[tuple, KernelSpec] = {}


def gen_split(karg: ir.KernelArg, name: str, rows: int, kdim: int, rows_p: int, k_p: int,
              row_var: str, k_var: str) -> KernelSpec:
    """``_gen_split`` memoised on the operand's value (a large proc asks for the
    same operand's split source many times while grouping and planning)."""
    import dataclasses
    key = (repr(karg), name, rows, kdim, rows_p, k_p, row_var, k_var)
    sp = _SPLIT_CACHE.get(key)
    if sp is None:
        if len(_SPLIT_CACHE) > 200000:
            _SPLIT_CACHE.clear()
        sp = _SPLIT_CACHE[key] = _gen_split(karg, name, rows, kdim, rows_p, k_p, row_var, k_var)
    return dataclasses.replace(sp, extra=dict(sp.extra))


def _gen_split(karg: ir.KernelArg, name: str, rows: int, kdim: int, rows_p: int, k_p: int,
               row_var: str, k_var: str) -> KernelSpec:
    """Gather operand(row, k) via its access expression into K-major hi/lo
    arrays (``rows_p`` x ``k_p``, zero-padded).  ``row_var``/``k_var`` say which
    of the reference's X/Y carries row and k.

    One 256-thread block per 64 x 64 tile.  The operand is read along the axis
    it is contiguous in (for a concatenation: the axis all of its pieces are
    contiguous in) with 16-byte loads where the access is aligned, and through
    a shared-memory transpose when that axis is the row axis; hi and lo are
    written with 16-byte stores."""
    bufs = sorted({codegen.view_of(km, set()) for km in codegen._kmats_of(karg)})
    rng = {"X": (0, max(rows, kdim)), "Y": (0, max(rows, kdim)), "G": (0, 0)}
    it = "int"
    for e in _karg_exprs(karg):
        if exprs.subexpr_max(e, rng) >= (1 << 31) - 64:
            it = "long long"
    if rows_p * k_p >= (1 << 31) - 64:
        it = "long long"
    em = Emitter(bufs, it)
    orient = "k"
    leaves = codegen._kmats_of(karg)
    plain = isinstance(karg, ir.KMatrix) and not karg.is_temp
    if leaves and len(leaves) == len(_leaves(karg)):
        if all(exprs.lanes(km.access, k_var, 4).s == 1 for km in leaves):
            orient = "k"
        elif all(exprs.lanes(km.access, row_var, 4).s == 1 for km in leaves):
            orient = "r"
    lane_var, other = (k_var, row_var) if orient == "k" else (row_var, k_var)
    vec = plain and exprs.lanes(karg.access, lane_var, 4, {other: 1}).unit(4)
    extent = kdim if orient == "k" else rows          # of the lane axis
    params = ", ".join([f"const float* __restrict__ p{i}" for i in range(len(bufs))] +
                       ["float* __restrict__ hi", "float* __restrict__ lo"])
    # one float4 of the lane axis at (ga, gb): ga = lane-axis start, gb = other coordinate
    coords = (lambda ga, gb: {k_var: ga, row_var: gb}) if orient == "k" else \
        (lambda ga, gb: {row_var: ga, k_var: gb})
    other_ext = rows if orient == "k" else kdim

    def uniform_cond(cond) -> bool:
        """Whether a concatenation's condition has one value over the four
        lanes of a float4 (``ga`` is a multiple of 4)."""
        gc = codegen._gt_const(cond)
        if gc is not None and exprs._var(gc[0]) == lane_var:
            t = gc[1]
            return float(t) == int(t) and (int(t) + 1) % 4 == 0
        return exprs.lanes(cond, lane_var, 4, {other: 1}).s == 0

    def tree4(k, dst: str, ga: str, gb: str, env0) -> List[str]:
        """Four lane values of ``k`` into ``dst``: a concatenation whose
        condition is the same for the four lanes branches once and reads the
        chosen piece (the piece the per-element conditionals select), a plain
        unit-stride piece with one 16-byte load."""
        if isinstance(k, ir.KConcat) and uniform_cond(k.condition):
            cp = codegen.concat_pieces(k)
            if cp is not None and all(uniform_cond(ir.Bin("MoreThan", cp[0], ir.Const(t))) for t in cp[2][1:]):
                # a chain of pieces along one axis: binary search over the thresholds
                v, parts, ths = cp

                def search(lo: int, hi: int) -> List[str]:
                    if hi - lo == 1:
                        return tree4(parts[lo], dst, ga, gb, env0)
                    mid = (lo + hi) // 2
                    return ([f"if ({em.expr(v, env0)} > ({it}){ths[mid]}) {{"] +
                            ["    " + x for x in search(mid, hi)] + ["} else {"] +
                            ["    " + x for x in search(lo, mid)] + ["}"])
                return search(0, len(parts))
            return ([f"if ({em.expr(k.condition, env0)} != 0) {{"] +
                    ["    " + x for x in tree4(k.karg_two, dst, ga, gb, env0)] + ["} else {"] +
                    ["    " + x for x in tree4(k.karg_one, dst, ga, gb, env0)] + ["}"])
        out = []
        kvec = isinstance(k, ir.KMatrix) and not k.is_temp and \
            exprs.lanes(k.access, lane_var, 4, {other: 1}).unit(4)
        if kvec:
            out.append(f"if ({ga} + 3 < ({it}){extent}) {dst} = "
                       f"*reinterpret_cast<const float4*>(&{em.at(k, env0)});")
            out.append("else {")
        else:
            out.append("{")
        for j, comp in enumerate("xyzw"):
            envj = dict(coords(f"({ga} + {j})", gb), G=f"(({it})0)")
            out.append(f"    if ({ga} + {j} < ({it}){extent}) {dst}.{comp} = {em.scalar_karg(k, envj, {})};")
        out.append("}")
        return out

    def load4(dst: str, ga: str, gb: str) -> str:
        if not plain and isinstance(karg, ir.KConcat) and uniform_cond(karg.condition):
            env0 = dict(coords(ga, gb), G=f"(({it})0)")
            lines = [f"float4 {dst} = make_float4(0.0f, 0.0f, 0.0f, 0.0f);",
                     f"if ({gb} < ({it}){other_ext}) {{"]
            lines += ["    " + x for x in tree4(karg, dst, ga, gb, env0)]
            lines.append("}")
            return "\n        ".join(lines)
        env0 = dict(coords(ga, gb), G=f"(({it})0)")
        lines = [f"float4 {dst} = make_float4(0.0f, 0.0f, 0.0f, 0.0f);",
                 f"if ({gb} < ({it}){other_ext}) {{"]
        if vec:
            lines.append(f"    if ({ga} + 3 < ({it}){extent}) {dst} = "
                         f"*reinterpret_cast<const float4*>(&{em.at(karg, env0)});")
            lines.append("    else {")
        else:
            lines.append("    {")
        for j, comp in enumerate("xyzw"):
            envj = dict(coords(f"({ga} + {j})", gb), G=f"(({it})0)")
            lines.append(f"        if ({ga} + {j} < ({it}){extent}) {dst}.{comp} = {em.scalar_karg(karg, envj, {})};")
        lines.append("    }")
        lines.append("}")
        return "\n        ".join(lines)

    split4 = """        unsigned h0, h1, h2, h3, l0, l1, l2, l3;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h0) : "f"(v.x));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h1) : "f"(v.y));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h2) : "f"(v.z));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h3) : "f"(v.w));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l0) : "f"(v.x - __uint_as_float(h0)));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l1) : "f"(v.y - __uint_as_float(h1)));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l2) : "f"(v.z - __uint_as_float(h2)));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l3) : "f"(v.w - __uint_as_float(h3)));
        *reinterpret_cast<float4*>(&hi[o]) = make_float4(__uint_as_float(h0), __uint_as_float(h1),
                                                         __uint_as_float(h2), __uint_as_float(h3));
        *reinterpret_cast<float4*>(&lo[o]) = make_float4(__uint_as_float(l0), __uint_as_float(l1),
                                                         __uint_as_float(l2), __uint_as_float(l3));"""
    if orient == "k":
        body = f"""    #pragma unroll
    for (int s = 0; s < 4; ++s) {{
        const int idx = threadIdx.x + s * 256, row = idx >> 4, kq = (idx & 15) * 4;
        const {it} gr = r0 + row, gk = k0 + kq;
        if (gk >= ({it}){k_p}) continue;
        {load4("v", "gk", "gr")}
        const {it} o = gr * ({it}){k_p} + gk;
{split4}
    }}"""
    else:
        body = f"""    __shared__ float t[64][65];
    #pragma unroll
    for (int s = 0; s < 4; ++s) {{
        const int idx = threadIdx.x + s * 256, kk = idx >> 4, rq = (idx & 15) * 4;
        const {it} gk = k0 + kk, gr = r0 + rq;
        {load4("u", "gr", "gk")}
        t[kk][rq] = u.x; t[kk][rq + 1] = u.y; t[kk][rq + 2] = u.z; t[kk][rq + 3] = u.w;
    }}
    __syncthreads();
    #pragma unroll
    for (int s = 0; s < 4; ++s) {{
        const int idx = threadIdx.x + s * 256, row = idx >> 4, kq = (idx & 15) * 4;
        const {it} gr = r0 + row, gk = k0 + kq;
        if (gk >= ({it}){k_p}) continue;
        const float4 v = make_float4(t[kq][row], t[kq + 1][row], t[kq + 2][row], t[kq + 3][row]);
        const {it} o = gr * ({it}){k_p} + gk;
{split4}
    }}"""
    src = f"""extern "C" __global__ void __launch_bounds__(256) {name}({params}) {{
    const {it} r0 = ({it})blockIdx.y * 64, k0 = ({it})blockIdx.x * 64;
{body}
}}
"""
    assert rows_p % 64 == 0 and k_p % 4 == 0
    return KernelSpec(name, src, bufs, (-(-k_p // 64), rows_p // 64, 1), (256, 1, 1), 0, "split",
                      4 * rows * kdim + 8 * rows_p * k_p)


def _leaves(k):
    if isinstance(k, ir.KConcat):
        return _leaves(k.karg_one) + _leaves(k.karg_two)
    return [k]


def _karg_exprs(k):
    if isinstance(k, ir.KMatrix) and not k.is_temp:
        return [k.access]
    if isinstance(k, ir.KConcat):
        return [k.condition] + _karg_exprs(k.karg_one) + _karg_exprs(k.karg_two)
    return []


# ---------------------------------------------------------------- gemm kernel

GEMM_TEMPLATE = r"""
struct __align__(64) TmapT { unsigned long long v[16]; };

#define AD_WAIT_NS 2000000000ull   // 2 s: far above any legitimate wait

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned cnt) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(b)), "r"(cnt));
}
__device__ __forceinline__ bool mbar_try(unsigned long long* b, unsigned phase) {
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(b)), "r"(phase) : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// bounded wait on an mbarrier phase: false after AD_WAIT_NS, or at once if another role aborted
__device__ __noinline__ bool mbar_wait(unsigned long long* b, unsigned phase, volatile int* abort_flag) {
    if (mbar_try(b, phase)) return true;
    const unsigned long long t0 = gtime();
    while (true) {
        for (int i = 0; i < 128; ++i)
            if (mbar_try(b, phase)) return true;
        if (*abort_flag) return false;
        if (gtime() - t0 > AD_WAIT_NS) return false;
    }
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const TmapT* map, unsigned long long* bar, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(smem_u32(dst)), "l"((unsigned long long)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ unsigned long long sdesc(const void* p) {
    // K-major, rows of ROWB bytes swizzled in 8-row atoms: start>>4, LBO=16B (unused),
    // SBO = 8 * ROWB, version 1, layout SWZ (2 = 128B swizzle, 4 = 64B swizzle)
    const unsigned long long a = (smem_u32(p) >> 4) & 0x3FFFull;
    return a | (1ull << 16) | ((8ull * ROWB >> 4) << 32) | (1ull << 46) | ((unsigned long long)SWZ << 61);
}
__device__ __forceinline__ void mma_tf32(unsigned tmem, unsigned long long ad, unsigned long long bd, unsigned idesc, unsigned acc) {
    asm volatile("{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}"
                 :: "r"(tmem), "l"(ad), "l"(bd), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void tmem_ld32(unsigned taddr, unsigned (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(unsigned taddr, const unsigned (&r)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
           "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
           "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
           "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tile_of_n(int t, int num_n, int& m_blk, int& n_blk) {
    // grouped raster: GROUP m-blocks share each sweep over n so A panels stay in L2
    constexpr int GROUP = GROUP_M, NUM_M = M_BLOCKS;
    const int per_group = GROUP * num_n;
    const int g = t / per_group, first = g * GROUP;
    const int gsz = (NUM_M - first) < GROUP ? (NUM_M - first) : GROUP;
    const int r = t % per_group;
    m_blk = first + r % gsz;
    n_blk = r / gsz;
}

DECODE_FN
// Persistent, warp-specialised: warp 0 = TMA producer, warp 1 = MMA issuer,
// warps 2..9 = epilogue (TMEM lane quarter = warp % 4, column half = (warp - 2) / 4).
// Two TMEM accumulators (2 x BN columns) let the epilogue of one tile overlap the
// MMAs of the next.
extern "C" __global__ void __launch_bounds__(320, 1) NAME(
    const __grid_constant__ TmapT tAh, const __grid_constant__ TmapT tAl,
    const __grid_constant__ TmapT tBh, const __grid_constant__ TmapT tBl,
    PARAMS int* __restrict__ err)
{
    constexpr int BN = TILE_N, STAGES = NSTAGES, KB = KBLOCKS, NUM_TILES = TOTAL_UNITS;
    constexpr unsigned A_BYTES = 128 * ROWB, B_BYTES = BN * ROWB;
    constexpr unsigned STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    constexpr int EPI_WARPS = 8;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((unsigned long long)smem_raw + 1023) & ~1023ull);
    float* trans = (float*)(smem + STAGES * STAGE_BYTES);                     // 8 warps x 32 x 32
    unsigned long long* full = (unsigned long long*)(trans + EPI_WARPS * 1024);
    unsigned long long* empty = full + STAGES;
    unsigned long long* tfull = empty + STAGES;
    unsigned long long* tempty = tfull + 2;
    unsigned long long* drain = tempty + 2;                                   // abort path only
    unsigned* tmem_slot = (unsigned*)(drain + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    volatile int* consumed = abort_flag + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], EPI_WARPS); }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *consumed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(2 * BN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int it = 0;
            for (int t = blockIdx.x; t < NUM_TILES && !*abort_flag; t += gridDim.x) {
                int inst, ks, mb, nb;
                decode(t, inst, ks, mb, nb);
                const int arow = A_ROW + mb * 128, brow = B_ROW + nb * BN;
                const int kb0 = ks * KB / KSPLIT, kb1 = (ks + 1) * KB / KSPLIT;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, abort_flag)) {
                        if (!*abort_flag) atomicExch(err, 1);
                        *abort_flag = 1;
                        break;
                    }
                    unsigned char* st = smem + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    tma_load_2d(st, &tAh, &full[s], kb * BKF, arow);
                    tma_load_2d(st + A_BYTES, &tAl, &full[s], kb * BKF, arow);
                    tma_load_2d(st + 2 * A_BYTES, &tBh, &full[s], kb * BKF, brow);
                    tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tBl, &full[s], kb * BKF, brow);
                }
            }
            if (*abort_flag) {
                // drain (bounded): copies issued but never consumed must land before exit
                for (int k = *consumed; k < it; ++k) {
                    const unsigned long long t0 = gtime();
                    while (!mbar_try(&full[k % STAGES], (k / STAGES) & 1) && gtime() - t0 < AD_WAIT_NS) {}
                }
            }
        }
#if AD_FOLD == 0
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer: D(128 x BN) += A(128 x 8) * B(BN x 8)^T, K-major, 3xTF32
            constexpr unsigned IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((unsigned)(BN >> 3) << 17) | ((128u >> 4) << 24);
            int it = 0, lt = 0;
            for (int t = blockIdx.x; t < NUM_TILES && !*abort_flag; t += gridDim.x, ++lt) {
                const int a = lt & 1;
                if (lt >= 2 && !mbar_wait(&tempty[a], ((lt >> 1) - 1) & 1, abort_flag)) {
                    if (!*abort_flag) atomicExch(err, 4);
                    *abort_flag = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const unsigned d = tmem + (unsigned)(a * BN);
                bool ok = true;
                int inst, ks, mb, nb;
                decode(t, inst, ks, mb, nb);
                const int kb0 = ks * KB / KSPLIT, kb1 = (ks + 1) * KB / KSPLIT;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) {
                        if (!*abort_flag) atomicExch(err, 2);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    unsigned char* st = smem + s * STAGE_BYTES;
                    const unsigned long long ah = sdesc(st), al = sdesc(st + A_BYTES);
                    const unsigned long long bh = sdesc(st + 2 * A_BYTES), bl = sdesc(st + 2 * A_BYTES + B_BYTES);
                    #pragma unroll
                    for (int k8 = 0; k8 < BKF / 8; ++k8) {
                        const unsigned long long adv = (unsigned long long)(k8 * 32) >> 4;  // 8 fp32 = 32 bytes
                        const unsigned first = (kb > kb0 || k8 > 0) ? 1u : 0u;
                        mma_tf32(d, ah + adv, bh + adv, IDESC, first);
                        mma_tf32(d, ah + adv, bl + adv, IDESC, 1u);
                        mma_tf32(d, al + adv, bh + adv, IDESC, 1u);
                    }
                    mma_commit(&empty[s]);
                    *consumed = it + 1;
                }
                if (!ok) break;
                mma_commit(&tfull[a]);
            }
            if (*abort_flag && it > 0) {
                // MMAs already issued may still be running: let them finish (bounded)
                // before the block frees its TMEM
                mma_commit(drain);
                const unsigned long long t0 = gtime();
                while (!mbar_try(drain, 0) && gtime() - t0 < AD_WAIT_NS) {}
            }
        }
    } else {
        // ---------------- epilogue warps
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;       // which half of the BN columns
        float* tr = trans + (warp - 2) * 1024;
        int lt = 0;
        for (int t = blockIdx.x; t < NUM_TILES; t += gridDim.x, ++lt) {
            const int a = lt & 1;
            if (!mbar_wait(&tfull[a], (lt >> 1) & 1, abort_flag)) {
                if (lane == 0 && !*abort_flag) atomicExch(err, 3);
                *abort_flag = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            int inst, ks, mb, nb;
            decode(t, inst, ks, mb, nb);
            const int m0 = mb * 128, n0 = nb * BN;
            EPI_PTRS
            #pragma unroll 1
            for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
                unsigned r[32];
                const unsigned taddr = tmem + ((unsigned)(q * 32) << 16) + (unsigned)(a * BN + c * 32);
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                      "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                      "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c == (half + 1) * (BN / 64) - 1) {
                    // last TMEM read of this tile by this warp: hand the accumulator back
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[a]);
                }
                #pragma unroll
                for (int j = 0; j < 32; ++j) tr[lane * 32 + (j ^ lane)] = __uint_as_float(r[j]);
                __syncwarp();
                // all 32 rows unrolled: the epilogue's global loads (bias, residuals,
                // in-place parameters) are issued together instead of 4 at a time
                CHUNK_SETUP
                #pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const IDX om = (IDX)m0 + q * 32 + i;
                    const IDX on = ON_BASE + lane;
                    if (CHUNK_OK && om < (IDX)M_DIM && on < (IDX)N_DIM) {
                        const float accv = tr[i * 32 + (lane ^ i)];
                        EPILOGUE
                    }
                }
                __syncwarp();
            }
        }
    }
#else
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer, folded accumulation: every AD_FOLD K blocks the
            // chunk accumulator (TMEM columns [0, BN)) is handed to the epilogue warps, which
            // add it into fp32 running sums (columns [BN, 2 BN)) on the CUDA cores
            constexpr unsigned IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((unsigned)(BN >> 3) << 17) | ((128u >> 4) << 24);
            int it = 0, gc = 0;
            for (int t = blockIdx.x; t < NUM_TILES && !*abort_flag; t += gridDim.x) {
                bool ok = true;
                int inst, ks, mb, nb;
                decode(t, inst, ks, mb, nb);
                const int kb0 = ks * KB / KSPLIT, kb1 = (ks + 1) * KB / KSPLIT;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const bool cstart = ((kb - kb0) % AD_FOLD) == 0;
                    if (cstart && gc > 0) {
                        // the previous chunk has been read out of the accumulator
                        if (!mbar_wait(&tempty[0], (gc - 1) & 1, abort_flag)) {
                            if (!*abort_flag) atomicExch(err, 4);
                            *abort_flag = 1;
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    }
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) {
                        if (!*abort_flag) atomicExch(err, 2);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    unsigned char* st = smem + s * STAGE_BYTES;
                    const unsigned long long ah = sdesc(st), al = sdesc(st + A_BYTES);
                    const unsigned long long bh = sdesc(st + 2 * A_BYTES), bl = sdesc(st + 2 * A_BYTES + B_BYTES);
                    #pragma unroll
                    for (int k8 = 0; k8 < BKF / 8; ++k8) {
                        const unsigned long long adv = (unsigned long long)(k8 * 32) >> 4;  // 8 fp32 = 32 bytes
                        const unsigned first = (!cstart || k8 > 0) ? 1u : 0u;
                        mma_tf32(tmem, ah + adv, bh + adv, IDESC, first);
                        mma_tf32(tmem, ah + adv, bl + adv, IDESC, 1u);
                        mma_tf32(tmem, al + adv, bh + adv, IDESC, 1u);
                    }
                    mma_commit(&empty[s]);
                    *consumed = it + 1;
                    if ((kb + 1 - kb0) % AD_FOLD == 0 || kb + 1 == kb1) {
                        mma_commit(&tfull[0]);
                        ++gc;
                    }
                }
                if (!ok) break;
            }
            if (*abort_flag && it > 0) {
                // MMAs already issued may still be running: let them finish (bounded)
                // before the block frees its TMEM
                mma_commit(drain);
                const unsigned long long t0 = gtime();
                while (!mbar_try(drain, 0) && gtime() - t0 < AD_WAIT_NS) {}
            }
        }
    } else {
        // ---------------- epilogue warps, folded accumulation
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;       // which half of the BN columns
        float* tr = trans + (warp - 2) * 1024;
        int egc = 0;
        bool live = true;
        for (int t = blockIdx.x; t < NUM_TILES && live; t += gridDim.x) {
            int inst, ks, mb, nb;
            decode(t, inst, ks, mb, nb);
            const int kb0 = ks * KB / KSPLIT, kb1 = (ks + 1) * KB / KSPLIT;
            const int nch = (kb1 - kb0 + AD_FOLD - 1) / AD_FOLD;
            const int m0 = mb * 128, n0 = nb * BN;
            const unsigned lanes = (unsigned)(q * 32) << 16;
            for (int ch = 0; ch < nch; ++ch, ++egc) {
                if (!mbar_wait(&tfull[0], egc & 1, abort_flag)) {
                    if (lane == 0 && !*abort_flag) atomicExch(err, 3);
                    *abort_flag = 1;
                    live = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if (ch + 1 < nch) {
                    // fold this chunk into the running sums: sum = (ch ? sum : 0) + chunk
                    #pragma unroll 1
                    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
                        unsigned r[32], u[32];
                        tmem_ld32(tmem + lanes + (unsigned)(c * 32), r);
                        if (ch > 0) {
                            tmem_ld32(tmem + lanes + (unsigned)(BN + c * 32), u);
                            #pragma unroll
                            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(u[j]) + __uint_as_float(r[j]));
                        }
                        tmem_st32(tmem + lanes + (unsigned)(BN + c * 32), r);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[0]);
                    continue;
                }
                // last chunk of the tile: sum + chunk, then the tile's epilogue
                EPI_PTRS
                #pragma unroll 1
                for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
                    unsigned r[32];
                    tmem_ld32(tmem + lanes + (unsigned)(c * 32), r);
                    if (nch > 1) {
                        unsigned u[32];
                        tmem_ld32(tmem + lanes + (unsigned)(BN + c * 32), u);
                        #pragma unroll
                        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(u[j]) + __uint_as_float(r[j]));
                    }
                    if (c == (half + 1) * (BN / 64) - 1) {
                        // last TMEM read of this chunk by this warp: hand the accumulator back
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[0]);
                    }
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) tr[lane * 32 + (j ^ lane)] = __uint_as_float(r[j]);
                    __syncwarp();
                    CHUNK_SETUP
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const IDX om = (IDX)m0 + q * 32 + i;
                        const IDX on = ON_BASE + lane;
                        if (CHUNK_OK && om < (IDX)M_DIM && on < (IDX)N_DIM) {
                            const float accv = tr[i * 32 + (lane ^ i)];
                            EPILOGUE
                        }
                    }
                    __syncwarp();
                }
            }
        }
    }
#endif
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(2 * BN) : "memory");
    }
}
"""


def choose_ksplit(units: int, kblocks: int, sm_count: int, bn: int = 256) -> int:
    """K slices per output tile: minimise waves x (K blocks per slice + pipeline
    fill), at least 4 K blocks per slice.  More than one slice adds the partial
    sums' round trip and the summing kernel's launch, about 8 us, charged in K
    blocks.  A K block takes ~0.43 us whatever the tile width up to 256 (the
    4096^3 product ran 1024 tiles of 128 x 128 at the same time per K block as
    512 tiles of 128 x 256): the stage pipeline, not the MMA, sets it, which is
    also why the widest tile is always used."""
    kblock_us = 0.43
    penalty = -(-8.0 // kblock_us)
    best, best_cost = 1, None
    for s_ in range(1, min(32, kblocks // 4) + 1):
        waves = -(-units * s_ // sm_count)
        cost = waves * (-(-kblocks // s_) + 6) + (penalty if s_ > 1 else 0)
        if best_cost is None or cost < best_cost:
            best, best_cost = s_, cost
    return best


DECODE_PLAIN = """__device__ __forceinline__ void decode(int t, int& inst, int& ks, int& m_blk, int& n_blk) {
    // instances of a grouped launch are consecutive ranges of KSPLIT x M_BLOCKS x N_BLOCKS
    // work units; ks = which slice of the K blocks this unit accumulates
    constexpr int PER = M_BLOCKS * N_BLOCKS;
    inst = t / (PER * KSPLIT);
    const int r = t - inst * (PER * KSPLIT);
    ks = r / PER;
    tile_of_n(r - ks * PER, N_BLOCKS, m_blk, n_blk);
}
"""

DECODE_SEG = """// segments: instances sharing one A operand whose B operands are consecutive rows
// of the stacked B, computed as one product over their concatenated columns
__constant__ int ad_seg_start[NSEG + 1] = {SEG_START};   // first work unit
__constant__ int ad_seg_nb[NSEG] = {SEG_NB};             // n-blocks
__constant__ int ad_seg_arow[NSEG] = {SEG_AROW};         // first row in the stacked A
__constant__ int ad_seg_brow[NSEG] = {SEG_BROW};         // first row in the stacked B
__constant__ int ad_seg_ncols[NSEG] = {SEG_NCOLS};       // instances x padded N
__constant__ int ad_seg_first[NSEG] = {SEG_FIRST};       // first instance (table row)
__device__ __forceinline__ void decode(int t, int& seg, int& ks, int& m_blk, int& n_blk) {
    int s = 0;
    while (s + 1 < NSEG && t >= ad_seg_start[s + 1]) ++s;
    const int r = t - ad_seg_start[s], per = M_BLOCKS * ad_seg_nb[s];
    seg = s;
    ks = r / per;
    tile_of_n(r - ks * per, ad_seg_nb[s], m_blk, n_blk);
}
"""


def gen_gemm(c, name: str, M: int, N: int, K: int, bn: int, stages: int, sm_count: int = 148,
             n_inst: int = 1, ksplit: int = 1, raw_out: bool = False, segments=None,
             np_stride: int = 0) -> KernelSpec:
    """The GEMM kernel of dot command ``c``.  With ``n_inst > 1`` it is a grouped
    launch over ``n_inst`` commands whose kernels differ only in their pointers:
    the kernel then takes a device table, per instance ``[A row base, B row base,
    epilogue pointers...]`` (row bases index the stacked split operands).
    With ``segments`` (list of ``(A row base, first instance, count)``), each
    segment's instances share A and own consecutive ``np_stride``-row blocks
    of the stacked B: the segment is one product over ``count * np_stride``
    columns with ``bn``-wide tiles, and every 32-column chunk of the epilogue
    finds its instance (N fusion of narrow per-head products).
    With ``ksplit > 1`` each output tile is computed as ``ksplit`` partial sums
    over consecutive K ranges, stored raw to ``ad_ws[inst][slice][M][N]``; the
    fused epilogue then runs in ``gen_splitk_epilogue``'s kernel; ``raw_out``
    does the same with one slice (epilogues too heavy for the GEMM's warps)."""
    rng = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    it = index_type(_epi_only(c), rng)
    bufs, em = codegen.make_emitter(c, it)
    tabw = 2 + len(bufs)
    raw = ksplit > 1 or raw_out
    ivar = "cinst" if segments else "inst"
    if not raw:
        epi = dot_epilogue(c, em, it, "accv", {"X": "om", "Y": "on", "G": f"(om * ({it}){N} + on)"})
        epi = "\n                        ".join(epi.split("\n"))
    else:
        epi = (f"ad_ws[((long long)({ivar} * {ksplit} + ks) * {M} + (long long)om) * {N} + (long long)on] = accv;")
    ptr_decls = lambda iv, ind: f"\n{ind}".join(
        f"float* __restrict__ p{i} = reinterpret_cast<float*>(ad_tab[(unsigned){iv} * {tabw}u + {2 + i}u]);"
        for i in range(len(bufs)))
    kb = pad(K, BK) // BKF
    mblk = pad(M, BM) // BM
    chunk_setup, on_base, chunk_ok = "", "(IDX)n0 + c * 32", "true"
    if segments:
        assert np_stride % 32 == 0 and n_inst > 1
        params = "const unsigned long long* __restrict__ ad_tab, " + ("float* __restrict__ ad_ws, " if raw else "")
        nbs = [-(-(cnt * np_stride) // bn) for _, _, cnt in segments]
        starts = [0]
        for nb_ in nbs:
            starts.append(starts[-1] + mblk * nb_ * ksplit)
        decode = (DECODE_SEG.replace("NSEG", str(len(segments)))
                  .replace("SEG_START", ", ".join(map(str, starts))).replace("SEG_NB", ", ".join(map(str, nbs)))
                  .replace("SEG_AROW", ", ".join(str(a) for a, _, _ in segments))
                  .replace("SEG_BROW", ", ".join(str(f * np_stride) for _, f, _ in segments))
                  .replace("SEG_NCOLS", ", ".join(str(cnt * np_stride) for _, _, cnt in segments))
                  .replace("SEG_FIRST", ", ".join(str(f) for _, f, _ in segments)))
        total = starts[-1]
        a_row, b_row, epi_ptrs = "ad_seg_arow[inst]", "ad_seg_brow[inst]", ""
        ind = "\n                "
        chunk_setup = (f"const int gcol = n0 + c * 32, cj = gcol / {np_stride};" + ind +
                       f"const bool chunk_ok = gcol < ad_seg_ncols[inst];" + ind +
                       f"const int cinst = ad_seg_first[inst] + (chunk_ok ? cj : 0);" +
                       ("" if raw else ind + ptr_decls("cinst", ind)))
        on_base, chunk_ok = f"(IDX)(gcol - cj * {np_stride})", "chunk_ok"
        nblk_plain = 1
    else:
        nblk_plain = pad(N, bn) // bn
        total = n_inst * mblk * nblk_plain * ksplit
        decode = DECODE_PLAIN
        if n_inst == 1:
            params = ("".join(f"float* __restrict__ p{i}, " for i in range(len(bufs))) if not raw
                      else "float* __restrict__ ad_ws, ")
            a_row, b_row, epi_ptrs = "0", "0", ""
        else:
            params = "const unsigned long long* __restrict__ ad_tab, " + ("float* __restrict__ ad_ws, " if raw else "")
            a_row = f"(int)ad_tab[(unsigned)inst * {tabw}u]"
            b_row = f"(int)ad_tab[(unsigned)inst * {tabw}u + 1u]"
            epi_ptrs = "" if raw else ptr_decls("inst", "\n            ")
    src = (GEMM_TEMPLATE.replace("DECODE_FN", decode).replace("NAME", name).replace("PARAMS", params)
           .replace("TILE_N", str(bn))
           .replace("NSTAGES", str(stages)).replace("KBLOCKS", str(kb)).replace("GROUP_M", str(GROUP_M))
           .replace("ROWB", str(BKF * 4)).replace("SWZ", "2" if BKF == 32 else "4").replace("BKF", str(BKF))
           .replace("TOTAL_UNITS", str(total)).replace("KSPLIT", str(ksplit))
           .replace("A_ROW", a_row).replace("B_ROW", b_row).replace("EPI_PTRS", epi_ptrs)
           .replace("CHUNK_SETUP", chunk_setup).replace("ON_BASE", on_base).replace("CHUNK_OK", chunk_ok)
           .replace("M_BLOCKS", str(mblk)).replace("N_BLOCKS", str(nblk_plain))
           .replace("IDX", it).replace("M_DIM", str(M)).replace("N_DIM", str(N)).replace("EPILOGUE", epi)
           .replace("AD_FOLD", str(fold_kb())))
    stage_bytes = 2 * 128 * BKF * 4 + 2 * bn * BKF * 4
    smem = stages * stage_bytes + 8 * 4096 + 1024 + 256
    grid = (min(total, sm_count), 1, 1)
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    epi_bytes = codegen.written_reads_bytes(_epi_only(c), rngw, {})
    if raw:
        bufs = []
        epi_bytes = 4 * ksplit * M * N
    spec = KernelSpec(name, src, bufs, grid, (320, 1, 1), smem, "gemm_tcgen05",
                      n_inst * (4 * (M * K + K * N) + epi_bytes), n_inst * 2 * M * N * K)
    spec.extra["tabw"] = tabw
    return spec


def gen_splitk_epilogue(c, name: str, M: int, N: int, ksplit: int, n_inst: int = 1) -> KernelSpec:
    """Sum the ``ksplit`` partial products of each output in slice order and run
    the command's fused epilogue (dp_elw_fuse.py:11-65 semantics).  Grouped: one
    ``blockIdx.z`` per instance, pointers from the GEMM's table."""
    rng = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    it = index_type(_epi_only(c), rng)
    bufs, em = codegen.make_emitter(c, it)
    tabw = 2 + len(bufs)
    epi = dot_epilogue(c, em, it, "accv", {"X": "om", "Y": "on", "G": f"(om * ({it}){N} + on)"})
    if n_inst == 1:
        params = "".join(f"float* __restrict__ p{i}, " for i in range(len(bufs)))
        ptrs = ""
    else:
        params = "const unsigned long long* __restrict__ ad_tab, "
        ptrs = "\n    ".join(
            f"float* __restrict__ p{i} = reinterpret_cast<float*>(ad_tab[(unsigned)inst * {tabw}u + {2 + i}u]);"
            for i in range(len(bufs)))
    epi = "\n        ".join(epi.split("\n"))
    # 4 outputs per thread, in four contiguous 256-output chunks per block: every load
    # instruction stays coalesced and each thread keeps 4x the loads in flight
    src = f"""extern "C" __global__ void __launch_bounds__(256) {name}({params}const float* __restrict__ ad_ws) {{
    const int inst = blockIdx.z;
    const long long base = (long long)blockIdx.x * 1024 + threadIdx.x;
    if (base >= {M * N}ll) return;
    {ptrs}
    const float* w = ad_ws + (long long)inst * {ksplit * M * N}ll;
    float accs[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j) {{
        const long long e = base + j * 256;
        float a = 0.0f;
        if (e < {M * N}ll) {{
            #pragma unroll
            for (int s = 0; s < {ksplit}; ++s) a += w[(long long)s * {M * N}ll + e];
        }}
        accs[j] = a;
    }}
    #pragma unroll
    for (int j = 0; j < 4; ++j) {{
        const long long e = base + j * 256;
        if (e >= {M * N}ll) break;
        const {it} om = ({it})(e / {N}), on = ({it})(e % {N});
        const float accv = accs[j];
        {epi}
    }}
}}
"""
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    epi_bytes = codegen.written_reads_bytes(_epi_only(c), rngw, {})
    spec = KernelSpec(name, src, bufs if n_inst == 1 else [], (-(-M * N // 1024), 1, n_inst), (256, 1, 1), 0,
                      "splitk_epilogue", n_inst * (4 * ksplit * M * N + epi_bytes))
    return spec


class _EpiView:
    """The epilogue chain of a dot command without the dot node itself."""

    def __init__(self, c):
        nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
        self.nodes = [n for n in nodes if type(n).__name__ != "DotProdNode"]
        dn = c if type(c).__name__ == "DotProdNode" else c.init_node
        self.nodes.append(ir.ContigiousNode(-1, [ir.KConstant(0.0)], dn.kres, dn.shape))


def _epi_only(c):
    v = _EpiView(c)
    return ir.ElwFuse(v.nodes, 0)


def plan(dev, cmd, name: str, sizes: Dict[int, int]) -> List[KernelSpec]:
    return plan_group(dev, [cmd], name, sizes)


class GroupPlan:
    """How one dot command, or a group of dot commands with identical kernels,
    runs on the tensor cores: instance order, distinct operands (commands
    reading the same data through the same access share one split), N-fused
    segments, tile width, K slices, and where the epilogue runs."""

    def __init__(self, cmds, sm_count: int = 148, name: str = "k"):
        dn, M, N, K = dot_shape(cmds[0])
        self.M, self.N, self.K = M, N, K
        bn0 = tile_n(N)
        self.Mp, self.Np, self.Kp = pad(M, BM), pad(N, bn0), pad(K, BK)
        sa, ia = self._dedupe(cmds, 0, name)
        # N fusion: narrow products (padded N below the widest tile) whose
        # instances each own a distinct B and share A with others
        self.segments = None
        n = len(cmds)
        if n > 1 and self.Np < 256:
            sb_try, ib_try = self._dedupe(cmds, 1, name)
            if len(sb_try) == n and len(sa) < n:
                order = sorted(range(n), key=lambda i: (ia[i], i))
                cmds = [cmds[i] for i in order]
                sa, ia = self._dedupe(cmds, 0, name)
                segs = []
                for i, a in enumerate(ia):
                    if segs and segs[-1][0] == a:
                        segs[-1][2] += 1
                    else:
                        segs.append([a, i, 1])
                self.segments = [(a * self.Mp, f, cnt) for a, f, cnt in segs]
        self.cmds = cmds
        self.sa, self.ia = sa, ia
        self.sb, self.ib = self._dedupe(cmds, 1, name)
        mblk = self.Mp // BM
        if self.segments:
            self.bn = tile_n(min(cnt for _, _, cnt in self.segments) * self.Np)
            units = sum(mblk * -(-(cnt * self.Np) // self.bn) for _, _, cnt in self.segments)
        else:
            self.bn = bn0
            units = n * mblk * (self.Np // bn0)
        self.ks = choose_ksplit(units, self.Kp // BKF, sm_count, self.bn)
        if os.environ.get("AD_GEMM_KSPLIT"):       # forced K slices (accuracy / tuning studies)
            self.ks = max(1, min(int(os.environ["AD_GEMM_KSPLIT"]), self.Kp // BKF))
        self.raw = self.ks > 1 or heavy_epilogue(cmds[0], n, units, self.Kp // BKF, sm_count)

    def _dedupe(self, cmds, which: int, name: str):
        rows, rows_p, rv, kv = ((self.M, self.Mp, "X", "Y") if which == 0 else (self.N, self.Np, "Y", "X"))
        specs, index, uniq = [], [], {}
        for c in cmds:
            sp = gen_split(dot_shape(c)[0].kargs[which], name + ("_splitA" if which == 0 else "_splitB"),
                           rows, self.K, rows_p, self.Kp, rv, kv)
            key = (sp.src, tuple(sp.buffers))
            if key not in uniq:
                uniq[key] = len(specs)
                specs.append(sp)
            index.append(uniq[key])
        return specs, index

    def scratch_bytes(self) -> int:
        """Stacked hi/lo operands, then the partial sums / raw products."""
        n = len(self.cmds)
        ws = 4 * n * self.ks * self.M * self.N if self.raw else 0
        return 2 * 4 * (len(self.sa) * self.Mp * self.Kp + len(self.sb) * self.Np * self.Kp) + ws + 4096


def group_scratch_bytes(cmds, sm_count: int = 148) -> int:
    return GroupPlan(cmds, sm_count).scratch_bytes()


def heavy_epilogue(c, n_inst: int, units: int, kblocks: int, sm_count: int) -> bool:
    """Run the fused epilogue as its own kernel when that is estimated faster.
    Inside the GEMM the epilogue warps (8 per SM) sustain ~1.5 TB/s (measured:
    the 4096 x 2048 x 512 FFN product with bias + ReLU takes 43 us for 67 MB of
    epilogue traffic), overlapped with the main loop; a separate kernel over
    the whole GPU streams ~5 TB/s but adds the raw product's round trip
    (8 bytes per output) and a launch.  Epilogues that read much more than the
    product (the sum of every head's input gradient fused into one head's dot)
    or short-K products with read-heavy epilogues (attention backward) go
    separate."""
    dn, M, N, K = dot_shape(c)
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    epi = n_inst * codegen.written_reads_bytes(_epi_only(c), rngw, {})
    main_us = -(-units // sm_count) * (kblocks + 6) * 0.43
    fused_us = max(main_us, epi / 1.5e6)
    sep_us = main_us + (epi + 8 * n_inst * M * N) / 5.0e6 + 8.0
    return sep_us < fused_us


_KSIG = re.compile(r'extern "C" __global__ void __launch_bounds__\(256\) (\w+)\(([^)]*)\)\s*\{')


def _split_pair(sa, sb, name: str, a_hi: int, a_lo: int, a_stride: int,
                b_hi: int, b_lo: int, b_stride: int) -> KernelSpec:
    """One launch splitting every distinct A operand and every distinct B
    operand.  A flat grid enumerates each operand's 32 x 32 tiles (A's
    operands first); pointers come from a device table (per operand: its
    views, then its hi and lo destinations).  Operand u of A goes to rows
    ``[u * rows_p, (u + 1) * rows_p)`` of the stacked hi/lo arrays, likewise B."""
    parts, calls, rows = [], [], []
    cbase, tbase = 0, 0
    for tag, specs, hi, lo, stride in (("a", sa, a_hi, a_lo, a_stride), ("b", sb, b_hi, b_lo, b_stride)):
        first = specs[0]
        m = _KSIG.search(first.src)
        fn = f"{name}_{tag}"
        width = len(first.buffers) + 2
        # pointers are read from the table where they are used: a concatenated
        # operand has one per piece, and only the selected piece's is needed
        body = first.src[m.end():].replace("blockIdx.x", "ad_bx").replace("blockIdx.y", "ad_by")
        body = re.sub(r"\bp(\d+)\[", r"((const float*)ad_t[\1])[", body)
        body = body.replace("hi[", f"((float*)ad_t[{width - 2}])[").replace("lo[", f"((float*)ad_t[{width - 1}])[")
        parts.append(first.src[:m.start()] + f"__device__ __forceinline__ void {fn}("
                     f"const unsigned long long* __restrict__ ad_t, unsigned ad_bx, unsigned ad_by) {{" + body)
        args = "t"
        n = len(specs)
        gx, gy = first.grid[0], first.grid[1]
        per = gx * gy
        calls.append(f"""    if (c < {cbase + n * per}u) {{
        const unsigned r = c - {cbase}u, u = r / {per}u, w = r - u * {per}u;
        const unsigned long long* t = tab + {tbase} + (unsigned long long)u * {width};
        {fn}({args}, w % {gx}u, w / {gx}u);
        return;
    }}""")
        for u, x in enumerate(specs):
            rows.append((x.buffers, False, [], [hi + u * stride, lo + u * stride]))
        cbase += n * per
        tbase += n * width
    src = "\n".join(parts) + f"""
extern "C" __global__ void __launch_bounds__(256) {name}(const unsigned long long* __restrict__ tab) {{
    const unsigned c = blockIdx.x;
{chr(10).join(calls)}
}}
"""
    assert sa[0].block == sb[0].block == (256, 1, 1)
    sp = KernelSpec(name, src, [], (cbase, 1, 1), sa[0].block, 0, "split",
                    sum(x.bytes_moved for x in sa) + sum(x.bytes_moved for x in sb))
    sp.extra["table"] = rows
    sp.extra["nparam"] = None
    return sp


def plan_group(dev, cmds, name: str, sizes: Dict[int, int]) -> List[KernelSpec]:
    """Split + GEMM launches for one dot command, or for a group of dot commands
    with identical kernels (same shapes, accesses and epilogue; different
    buffers) as one grouped launch each."""
    from . import runtime as rt
    sm = dev.ctx.sm_count
    gp = GroupPlan(cmds, sm, name)
    cmds = gp.cmds
    M, N, K, Mp, Np, Kp, bn = gp.M, gp.N, gp.K, gp.Mp, gp.Np, gp.Kp, gp.bn
    nA, nB, n = len(gp.sa), len(gp.sb), len(cmds)
    base = dev.scratch_base
    a_hi, a_lo = base, base + 4 * nA * Mp * Kp
    b_hi = a_lo + 4 * nA * Mp * Kp
    b_lo = b_hi + 4 * nB * Np * Kp
    ws = b_lo + 4 * nB * Np * Kp
    assert gp.scratch_bytes() <= dev.scratch_bytes
    split = _split_pair(gp.sa, gp.sb, name + "_split", a_hi, a_lo, 4 * Mp * Kp, b_hi, b_lo, 4 * Np * Kp)
    g = gen_gemm(cmds[0], name + ("_tc" if n == 1 else "_tcx"), M, N, K, bn, stages_for(bn), sm, n,
                 gp.ks, gp.raw, gp.segments, Np)
    sw = BKF * 4
    maps = [rt.tmap_2d(a_hi, nA * Mp, Kp, 4 * Kp, 128, BKF, 4, sw), rt.tmap_2d(a_lo, nA * Mp, Kp, 4 * Kp, 128, BKF, 4, sw),
            rt.tmap_2d(b_hi, nB * Np, Kp, 4 * Kp, bn, BKF, 4, sw), rt.tmap_2d(b_lo, nB * Np, Kp, 4 * Kp, bn, BKF, 4, sw)]
    g.extra["prefix"] = [ctypes.create_string_buffer(m, 128) for m in maps]
    g.extra["suffix"] = ([ctypes.c_uint64(ws)] if gp.raw else []) + [ctypes.c_uint64(dev.err_ptr)]
    specs = [split, g]
    rows = []
    if n > 1:
        for i, c in enumerate(cmds):
            bufs, _ = codegen.make_emitter(c, "int")
            rows.append((bufs, False, [gp.ia[i] * Mp, gp.ib[i] * Np], []))
        g.buffers = []
        g.extra["table"] = rows
        g.extra["nparam"] = g.extra["tabw"]
    if gp.raw:
        e = gen_splitk_epilogue(cmds[0], name + ("_ske" if n == 1 else "_skex"), M, N, gp.ks, n)
        e.extra["suffix"] = [ctypes.c_uint64(ws)]
        if n > 1:
            e.extra["table"] = rows
            e.extra["nparam"] = g.extra["tabw"]
        specs.append(e)
    return specs


# ---------------------------------------------------------------- tensor-pipe peak probe

PROBE_TEMPLATE = r"""
extern "C" __global__ void __launch_bounds__(128, 1) tf32_probe(int iters, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((unsigned long long)smem_raw + 1023) & ~1023ull);
    unsigned long long* bar = (unsigned long long*)(smem + 3 * 32768);
    unsigned* tmem_slot = (unsigned*)(bar + 1);
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 3 * 32768 / 4; i += 128) ((float*)smem)[i] = 0.0f;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"((unsigned)__cvta_generic_to_shared(bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;"
                     :: "r"((unsigned)__cvta_generic_to_shared(tmem_slot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = *tmem_slot;
    if (threadIdx.x == 0) {
        constexpr unsigned IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
        const unsigned long long base = (unsigned long long)(((unsigned)__cvta_generic_to_shared(smem)) >> 4) & 0x3FFFull;
        const unsigned long long ad = base | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
        const unsigned long long bd = ad + (16384ull >> 4);
        for (int i = 0; i < iters; ++i) {
            const unsigned long long adv = (unsigned long long)((i & 3) * 32) >> 4;
            asm volatile("{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
                         " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}"
                         :: "r"(tmem), "l"(ad + adv), "l"(bd + adv), "r"(IDESC), "r"((unsigned)(i > 0)) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     :: "r"((unsigned)__cvta_generic_to_shared(bar)) : "memory");
    }
    __syncwarp();
    unsigned ok = 0;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(ok) : "r"((unsigned)__cvta_generic_to_shared(bar)) : "memory");
        if (ok) break;
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) { atomicExch(err, 4); break; }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" :: "r"(tmem) : "memory");
}
"""


def measure_tf32_peak(ctx, err_ptr: int, iters: int = 4096, reps: int = 5) -> float:
    """Dense kind::tf32 tensor-pipe throughput (TFLOP/s) with operands resident in
    shared memory: one CTA per SM issuing back-to-back 128x256x8 MMAs."""
    from . import runtime as rt
    cub = rt.compile_cubin(PROBE_TEMPLATE, "tf32_probe.cu")
    k = ctx.load(cub, "tf32_probe")
    smem = 3 * 32768 + 2048
    k.set_smem(smem)
    it = ctypes.c_int(iters)
    ep = ctypes.c_uint64(err_ptr)
    argv = (ctypes.c_void_p * 2)(ctypes.addressof(it), ctypes.addressof(ep))
    grid = (ctx.sm_count, 1, 1)
    ctx.launch(k, grid, (128, 1, 1), smem, argv, 0)
    ctx.sync()
    e0, e1 = ctx.event(True), ctx.event(True)
    e0.record(0)
    for _ in range(reps):
        ctx.launch(k, grid, (128, 1, 1), smem, argv, 0)
    e1.record(0)
    e1.sync()
    ms = e0.elapsed_ms(e1) / reps
    flops = ctx.sm_count * iters * 2.0 * 128 * 256 * 8
    return flops / (ms / 1e3) / 1e12
