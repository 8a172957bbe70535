.version 8.0
.target sm_89
.address_size 64

.visible .entry k_attention_causal(
        .param .u64 p_q,
        .param .u64 p_k,
        .param .u64 p_v,
        .param .u64 p_out
)
{
        .reg .pred %p<3>;
        .reg .f32  %f<33>;
        .reg .b16  %h<1>;
        .reg .f64  %d<1>;
        .reg .b32  %r<60>;
        .reg .b64  %rd<17>;

        ld.param.u64 %rd1, [p_q];
        cvta.to.global.u64 %rd2, %rd1;
        ld.param.u64 %rd3, [p_k];
        cvta.to.global.u64 %rd4, %rd3;
        ld.param.u64 %rd5, [p_v];
        cvta.to.global.u64 %rd6, %rd5;
        ld.param.u64 %rd7, [p_out];
        cvta.to.global.u64 %rd8, %rd7;
        mov.u32 %r1, %tid.x;
        and.b32 %r2, %r1, 31;
        shr.u32 %r3, %r1, 5;
        mov.u32 %r4, %ctaid.x;
        mad.lo.u32 %r5, %r4, 256, %r1;
        setp.ge.u32 %p1, %r5, 122880;
        @%p1 bra TILE_END_1;
        div.s32 %r6, %r5, 40960;
        div.s32 %r7, %r5, 8192;
        rem.s32 %r8, %r7, 5;
        div.s32 %r9, %r5, 32;
        rem.s32 %r10, %r9, 256;
        rem.s32 %r11, %r5, 32;
        mul.lo.s32 %r12, %r6, 81920;
        mul.lo.s32 %r13, %r8, 16384;
        add.s32 %r14, %r12, %r13;
        mul.lo.s32 %r15, %r10, 64;
        add.s32 %r16, %r14, %r15;
        mov.s32 %r17, 2;
        mul.lo.s32 %r18, %r11, %r17;
        add.s32 %r19, %r16, %r18;
        mul.wide.s32 %rd9, %r19, 4;
        add.s64 %rd10, %rd2, %rd9;
        ld.global.v2.f32 {%f1, %f2}, [%rd10];
        mov.f32 %f3, 0f3E000000;
        mov.f32 %f4, 0fFF800000;
        mov.f32 %f5, 0f00000000;
        mov.f32 %f6, 0f00000000;
        mov.f32 %f7, 0f00000000;
        mov.s32 %r20, 0;
        mov.s32 %r21, %r20;
        mov.s32 %r22, 1;
        mov.s32 %r23, 1;
        add.s32 %r24, %r10, %r23;
SL_2:
        setp.ge.s32 %p2, %r21, %r24;
        @%p2 bra SL_END_3;
        mul.lo.s32 %r25, %r6, 81920;
        mul.lo.s32 %r26, %r8, 16384;
        add.s32 %r27, %r25, %r26;
        mul.lo.s32 %r28, %r21, 64;
        add.s32 %r29, %r27, %r28;
        mov.s32 %r30, 2;
        mul.lo.s32 %r31, %r11, %r30;
        add.s32 %r32, %r29, %r31;
        mul.wide.s32 %rd11, %r32, 4;
        add.s64 %rd12, %rd4, %rd11;
        ld.global.v2.f32 {%f8, %f9}, [%rd12];
        mul.f32 %f10, %f1, %f8;
        mul.f32 %f11, %f2, %f9;
        add.f32 %f12, %f10, %f11;
        mov.f32 %f13, %f12;
        activemask.b32 %r33;
        mov.b32 %r34, %f13;
        shfl.sync.bfly.b32 %r35, %r34, 16, 0x1f, %r33;
        mov.b32 %f14, %r35;
        add.f32 %f13, %f13, %f14;
        mov.b32 %r36, %f13;
        shfl.sync.bfly.b32 %r37, %r36, 8, 0x1f, %r33;
        mov.b32 %f15, %r37;
        add.f32 %f13, %f13, %f15;
        mov.b32 %r38, %f13;
        shfl.sync.bfly.b32 %r39, %r38, 4, 0x1f, %r33;
        mov.b32 %f16, %r39;
        add.f32 %f13, %f13, %f16;
        mov.b32 %r40, %f13;
        shfl.sync.bfly.b32 %r41, %r40, 2, 0x1f, %r33;
        mov.b32 %f17, %r41;
        add.f32 %f13, %f13, %f17;
        mov.b32 %r42, %f13;
        shfl.sync.bfly.b32 %r43, %r42, 1, 0x1f, %r33;
        mov.b32 %f18, %r43;
        add.f32 %f13, %f13, %f18;
        mul.f32 %f19, %f13, %f3;
        mov.f32 %f20, %f4;
        max.f32 %f4, %f4, %f19;
        sub.f32 %f21, %f20, %f4;
        mul.f32 %f22, %f21, 0f3FB8AA3B;
        ex2.approx.f32 %f23, %f22;
        sub.f32 %f24, %f19, %f4;
        mul.f32 %f25, %f24, 0f3FB8AA3B;
        ex2.approx.f32 %f26, %f25;
        mul.f32 %f5, %f5, %f23;
        add.f32 %f5, %f5, %f26;
        mul.lo.s32 %r44, %r6, 81920;
        mul.lo.s32 %r45, %r8, 16384;
        add.s32 %r46, %r44, %r45;
        mul.lo.s32 %r47, %r21, 64;
        add.s32 %r48, %r46, %r47;
        mov.s32 %r49, 2;
        mul.lo.s32 %r50, %r11, %r49;
        add.s32 %r51, %r48, %r50;
        mul.wide.s32 %rd13, %r51, 4;
        add.s64 %rd14, %rd6, %rd13;
        ld.global.v2.f32 {%f27, %f28}, [%rd14];
        mul.f32 %f6, %f6, %f23;
        mul.f32 %f29, %f26, %f27;
        add.f32 %f6, %f6, %f29;
        mul.f32 %f7, %f7, %f23;
        mul.f32 %f30, %f26, %f28;
        add.f32 %f7, %f7, %f30;
        add.s32 %r21, %r21, %r22;
        bra SL_2;
SL_END_3:
        div.rn.f32 %f31, %f6, %f5;
        div.rn.f32 %f32, %f7, %f5;
        mul.lo.s32 %r52, %r6, 81920;
        mul.lo.s32 %r53, %r8, 16384;
        add.s32 %r54, %r52, %r53;
        mul.lo.s32 %r55, %r10, 64;
        add.s32 %r56, %r54, %r55;
        mov.s32 %r57, 2;
        mul.lo.s32 %r58, %r11, %r57;
        add.s32 %r59, %r56, %r58;
        mul.wide.s32 %rd15, %r59, 4;
        add.s64 %rd16, %rd8, %rd15;
        st.global.v2.f32 [%rd16], {%f31, %f32};
TILE_END_1:
        ret;
}
